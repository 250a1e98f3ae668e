"""Byte-parity cases on the benchmark configurations' own tables.

Each case builds, on the CPU and from a fixed seed, a cut-down batch of one benchmark
configuration (fewer and shorter streams) with that configuration's exact tables:

* ``laplace64``: the 64 Laplace tables over 256 symbols, rans64 push + bisection pop;
* ``gaussian_latent`` / ``gaussian_latent_escapes``: the 64 Gaussian scale tables (rows of up to
  ~3,100 entries, escape slot, offsets -t_k), rans32 with 8-bit words, escape coding on; the
  second case replaces 1 % of the symbols by values beyond their table's tail, so escapes are coded;
* ``zipf_alias`` / ``zipf_plain``: the Zipf(1.1) table over 4,096 symbols at fp 15, rans32_16, with
  alias tables at symbol precision 12 (built by the reference's own ``rans_alias_build_table``)
  and with plain push + bisection pop;
* ``mixture_invcdf``: the 256 two-Gaussian mixture tables over 1,024 symbols with their
  65,536-entry inverse-cdf rows, rans64 push + inverse-cdf pop;
* ``ragged_adaptive``: streams of lognormal lengths, one 33-entry cdf row per symbol; the
  reference codes each stream alone (B = 1, indexes arange(n)).

``tests/golden/make_config_golden.py`` runs the reference CPU path (oracle/_ref) on every case and
stores, per stream, the row length and a SHA-256 of the payload bytes, plus a digest of the inputs
(``tests/golden/config_cases.json``).  The CPU tests check the oracle against those records and
the GPU tests check the CUDA path against them.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "config_cases.json")


@dataclass
class Case:
    name: str
    builder: str
    kwargs: Dict[str, object] = field(default_factory=dict)


CASES: List[Case] = [
    Case("laplace64", "laplace64", dict(scale=1 / 4, length_scale=1 / 16)),
    Case("gaussian_latent", "gaussian_latent", dict(scale=1 / 8)),
    Case("gaussian_latent_escapes", "gaussian_latent", dict(scale=1 / 8, outliers=0.01)),
    Case("zipf_alias", "zipf_alias", dict(scale=1 / 128, length_scale=1 / 64)),
    Case("zipf_plain", "zipf_alias", dict(scale=1 / 128, length_scale=1 / 64, alias=False)),
    Case("mixture_invcdf", "mixture_invcdf", dict(scale=1 / 512, length_scale=1 / 32)),
    Case("ragged_adaptive", "ragged_adaptive", dict(scale=1 / 512, length_scale=1 / 64)),
]


def by_name(name: str) -> Case:
    return next(c for c in CASES if c.name == name)


def build(case: Case, alias_builder=None):
    """The case's inputs on the CPU (alias tables from `alias_builder`, the reference's own when
    the fixtures are made)."""
    from torch_ans_b200 import workloads as W
    kw = dict(case.kwargs)
    if case.builder == "zipf_alias":
        kw["alias_builder"] = alias_builder
    return W.BUILDERS[case.builder](device="cpu", **kw)


def _digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        a = np.ascontiguousarray(t.cpu().numpy() if isinstance(t, torch.Tensor) else t)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def input_digest(w) -> str:
    """Digest of everything the coder reads (symbols, indexes or row starts, every table)."""
    if hasattr(w, "row_starts"):
        return _digest(w.symbols, w.row_starts, w.cdfs, w.cdfs_sizes, w.offsets)
    return _digest(w.symbols, w.indexes, w.tables_for_push(), w.tables_for_pop(), w.cdfs_sizes, w.offsets)


def rows_record(stream: np.ndarray) -> Dict[str, object]:
    """Width, length column and per-row payload SHA-256 of a stream matrix."""
    s = np.ascontiguousarray(stream, dtype=np.int32)
    return {"width": int(s.shape[1]), "lengths": [int(x) for x in s[:, 0]],
            "payload_sha256": [hashlib.sha256(s[b, 1:].tobytes()[: int(s[b, 0])]).hexdigest()
                               for b in range(s.shape[0])]}


def ragged_stream_inputs(w, b):
    """Stream b of a ragged workload as the reference takes it alone: (1, n) symbols, indexes
    arange(n), its n cdf rows with sizes and offsets."""
    lo, hi = int(w.row_starts[b]), int(w.row_starts[b + 1])
    n = hi - lo
    return (w.symbols[lo:hi].reshape(1, n).contiguous(), torch.arange(n, dtype=torch.int32).reshape(1, n),
            w.cdfs[lo:hi].contiguous(), w.cdfs_sizes[lo:hi].contiguous(), w.offsets[lo:hi].contiguous())


def load_fixture() -> Dict[str, dict]:
    with open(FIXTURE) as f:
        return json.load(f)


def reference_record(case: Case, ref) -> dict:
    """Run the compiled reference (a module with the reference's `_C` surface, on CPU tensors)
    on a case and return its record."""
    w = build(case, alias_builder=ref.rans_alias_build_table)
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    rec = {"builder": case.builder, "kwargs": case.kwargs, "variant": w.variant, "input_sha256": input_digest(w)}
    if hasattr(w, "row_starts"):
        rows, popped = [], []
        for b in range(w.num_streams):
            sym, idx, cdf, sz, off = ragged_stream_inputs(w, b)
            st = getattr(ref, f"{w.variant}_init_stream")(1)
            getattr(ref, f"{w.variant}_push")(st, sym, idx, cdf, sz, off, **kw)
            rows.append(rows_record(st.numpy()))
            dec = getattr(ref, f"{w.variant}_pop")(st, idx, cdf, sz, off, **kw)
            assert torch.equal(dec, sym), (case.name, b)
            popped.append(rows_record(st.numpy()))
        rec.update(streams=w.num_streams, symbols=w.num_symbols,
                   per_stream=[{"width": r["width"], "length": r["lengths"][0], "payload_sha256": r["payload_sha256"][0]}
                               for r in rows],
                   popped=[{"length": p["lengths"][0], "payload_sha256": p["payload_sha256"][0]} for p in popped])
        return rec
    B = w.symbols.shape[0]
    st = getattr(ref, f"{w.variant}_init_stream")(B)
    getattr(ref, w.push_op)(st, w.symbols, w.indexes, w.tables_for_push(), w.cdfs_sizes, w.offsets, **kw)
    pushed = rows_record(st.numpy())
    dec = getattr(ref, w.pop_op)(st, w.indexes, w.tables_for_pop(), w.cdfs_sizes, w.offsets, **kw)
    assert torch.equal(dec, w.symbols), case.name
    rec.update(push_op=w.push_op, pop_op=w.pop_op, streams=B, symbols=int(w.symbols.numel()), pushed=pushed,
               popped=rows_record(st.numpy()),
               escapes_coded=bool(w.bypass and (w.symbols.numel() > 0) and _any_escape(w)))
    if case.builder == "zipf_alias" and case.kwargs.get("alias", True):
        rec["alias_tables_sha256"] = _digest(w.tables_for_push(), w.tables_for_pop())
    return rec


def _any_escape(w) -> bool:
    """Whether any symbol of the batch takes the escape path (value outside its table's range)."""
    v = w.symbols.to(torch.int64) - w.offsets.to(torch.int64)[w.indexes.to(torch.int64)]
    top = (w.cdfs_sizes.to(torch.int64) - 2)[w.indexes.to(torch.int64)]
    return bool(((v < 0) | (v >= top)).any())
