"""Write the golden vectors in tests/golden/ by running the REFERENCE torch_ans CPU path.

The reference has no golden compressed-byte vectors of its own (its coding tests are round trips,
tests/torch_ans_test.py:108-150), so byte-level parity is pinned here by running the reference
itself: its CPU extension compiled from its own sources by ``oracle/build_ref.py`` into
``oracle/_ref``.  Each case stores seeded inputs and the reference's outputs; the CPU test suite
then checks that ``oracle/rans_oracle.c`` reproduces every byte, and the GPU tests check the CUDA
path against the same files.

Inputs follow the reference's own test recipes: ``_generate_rans_params`` (pmf ~ randint(1,1024)
plus a tail of 1, quantised with rans_pmf_to_quantized_cdf, cdf_size = A + 2, offsets ~
randint(-8, 8); tests/torch_ans_test.py:14-29) so escape coding is hit on both sides, plus
bypass-off Laplace-like tables, inverse-cdf rows, alias tables, the 4-way interleaved format,
pushes onto non-empty streams with partial pops, and edge shapes (1 symbol, odd lengths,
single-symbol alphabets, large escape values).

Run where the reference checkout exists ($TORCH_ANS_REFERENCE, or ``reference`` beside this
repository):
    python oracle/build_ref.py && python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

REF = None


def ref():
    global REF
    if REF is None:
        build_ref.build()
        REF = build_ref.load()
        if REF is None:
            raise SystemExit("compiled reference not available (run oracle/build_ref.py)")
    return REF


def gen_params(g, num_dists, num_symbols, fp):
    """tests/torch_ans_test.py:14-29 recipe (seeded)."""
    pmfs = torch.randint(1, 1024, (num_dists, num_symbols), generator=g).float()
    pmfs = torch.cat([pmfs, torch.ones(num_dists, 1)], dim=1)
    pmfs = pmfs / pmfs.sum(dim=-1, keepdim=True)
    cdfs = ref().rans_pmf_to_quantized_cdf(pmfs, precision=fp)
    sizes = torch.full((num_dists,), num_symbols + 2, dtype=torch.int32)
    offsets = torch.randint(-8, 8, (num_dists,), generator=g, dtype=torch.int32)
    return cdfs, sizes, offsets


def laplace_tables(g, num_dists, alphabet, fp):
    """Bypass-off tables: discretised Laplace rows with every frequency >= 1 (exact integer
    quantiser: largest-remainder rounding of (2^fp - A) extra counts)."""
    rows = []
    x = torch.arange(alphabet, dtype=torch.float64) - alphabet // 2
    for _ in range(num_dists):
        scale = float(torch.exp(torch.empty(1, dtype=torch.float64).uniform_(np.log(0.3), np.log(8.0), generator=g)))
        p = torch.exp(-x.abs() / scale)
        p = p / p.sum()
        extra = (1 << fp) - alphabet
        want = p * extra
        base = torch.floor(want).long()
        rem = extra - int(base.sum())
        order = torch.argsort(want - base, descending=True)
        base[order[:rem]] += 1
        freq = base + 1
        cdf = torch.zeros(alphabet + 1, dtype=torch.long)
        cdf[1:] = torch.cumsum(freq, 0)
        rows.append(cdf)
    cdfs = torch.stack(rows).int()
    sizes = torch.full((num_dists,), alphabet + 1, dtype=torch.int32)
    return cdfs, sizes


def sample_from(g, cdfs, sizes, indexes, fp):
    """Symbols drawn from each row's pmf (values in [0, cdf_size-2], i.e. never the last slot
    unless it has mass)."""
    u = torch.randint(0, 1 << fp, indexes.shape, generator=g, dtype=torch.int64)
    rows = cdfs.long()[indexes.long()]
    return (torch.searchsorted(rows, u.unsqueeze(-1), right=True).squeeze(-1) - 1).int()


def inv_rows(cdfs, fp):
    r = torch.arange(1 << fp)
    inv = torch.stack([torch.searchsorted(c.sort().values, r, right=True) - 1 for c in cdfs.long()]).int()
    return torch.cat([cdfs, inv], dim=1)


CASES = {}


def add(name, **arrays):
    CASES[name] = arrays


def stream_bytes(stream):
    return np.frombuffer(b"".join(ref().rans_stream_to_byte_strings(stream)), np.uint8)


def run_coding(name, variant, symbols, indexes, cdfs, sizes, offsets, fp, bypass, bp=4,
               lookup="search", interleave=1, push_cdfs=None, pop_cdfs=None, prealloc=0):
    R = ref()
    init = getattr(R, f"{variant}_init_stream")
    stream = init(symbols.shape[0], interleave, prealloc)
    stream_in = stream.clone()
    if interleave == 4:
        push_fn = getattr(R, f"{variant}_i4_push")
    elif push_cdfs is not None:
        push_fn = getattr(R, f"{variant}_alias_push")
    else:
        push_fn = getattr(R, f"{variant}_push")
    pcdfs = push_cdfs if push_cdfs is not None else cdfs
    push_fn(stream, symbols, indexes, pcdfs, sizes, offsets, freq_precision=fp, bypass_coding=bypass,
            bypass_precision=bp)
    pushed = stream.clone()
    if lookup == "alias":
        pop_fn = getattr(R, f"{variant}_alias_pop")
    elif lookup == "invcdf":
        pop_fn = getattr(R, f"{variant}_i4_invcdf_pop" if interleave == 4 else f"{variant}_invcdf_pop")
    else:
        pop_fn = getattr(R, f"{variant}_i4_pop" if interleave == 4 else f"{variant}_pop")
    qcdfs = pop_cdfs if pop_cdfs is not None else cdfs
    st2 = R.rans_byte_strings_to_stream(R.rans_stream_to_byte_strings(stream))
    decoded = pop_fn(st2, indexes, qcdfs, sizes, offsets, freq_precision=fp, bypass_coding=bypass,
                     bypass_precision=bp)
    meta = dict(variant=variant, fp=fp, bypass=int(bypass), bp=bp, lookup=lookup,
                interleave=interleave, alias_push=int(push_cdfs is not None), prealloc=prealloc)
    add(name, meta=np.array(json.dumps(meta)), stream_in=stream_in.numpy(), symbols=symbols.numpy(),
        indexes=indexes.numpy(), cdfs=cdfs.numpy(), sizes=sizes.numpy(), offsets=offsets.numpy(),
        push_cdfs=(pcdfs.numpy()), pop_cdfs=qcdfs.numpy(), pushed=pushed.numpy(),
        pushed_bytes=stream_bytes(pushed), decoded=decoded.numpy(), popped=st2.numpy())
    assert (decoded == symbols).all(), name


def main():
    g = torch.Generator().manual_seed(20241201)
    fps = {"rans64": 16, "rans32": 16, "rans32_16": 15}
    for variant in ("rans64", "rans32", "rans32_16"):
        fp = fps[variant]
        # escape coding on both sides (reference test recipe, smaller)
        K, A, B, N = 4, 30, 5, 257
        cdfs, sizes, offsets = gen_params(g, K, A, fp)
        sym = torch.randint(-6, A + 12, (B, N), generator=g, dtype=torch.int32)
        idx = torch.randint(0, K, (B, N), generator=g, dtype=torch.int32)
        run_coding(f"{variant}_bypass", variant, sym, idx, cdfs, sizes, offsets, fp, True)
        run_coding(f"{variant}_bypass_invcdf", variant, sym, idx, cdfs, sizes, offsets, fp, True,
                   lookup="invcdf", pop_cdfs=inv_rows(cdfs, fp))
        run_coding(f"{variant}_i4_bypass", variant, sym, idx, cdfs, sizes, offsets, fp, True, interleave=4)
        if variant != "rans64":
            run_coding(f"{variant}_i4_invcdf", variant, sym, idx, cdfs, sizes, offsets, fp, True,
                       interleave=4, lookup="invcdf", pop_cdfs=inv_rows(cdfs, fp))
        # larger escape values at bypass precision 2 and 5
        big = torch.randint(-3000, 3000, (2, 64), generator=g, dtype=torch.int32)
        bidx = torch.randint(0, K, (2, 64), generator=g, dtype=torch.int32)
        run_coding(f"{variant}_bypass_bp2", variant, big, bidx, cdfs, sizes, offsets, fp, True, bp=2)
        run_coding(f"{variant}_bypass_bp5", variant, big, bidx, cdfs, sizes, offsets, fp, True, bp=5)
        # bypass off, peaky tables, zero offsets
        lc, ls = laplace_tables(g, 6, 64, fp)
        lo = torch.zeros(6, dtype=torch.int32)
        B2, N2 = 7, 403
        lidx = torch.randint(0, 6, (B2, N2), generator=g, dtype=torch.int32)
        lsym = sample_from(g, lc, ls, lidx, fp)
        run_coding(f"{variant}_plain", variant, lsym, lidx, lc, ls, lo, fp, False)
        run_coding(f"{variant}_plain_invcdf", variant, lsym, lidx, lc, ls, lo, fp, False,
                   lookup="invcdf", pop_cdfs=inv_rows(lc, fp))
        run_coding(f"{variant}_i4_plain", variant, lsym, lidx, lc, ls, lo, fp, False, interleave=4)
        run_coding(f"{variant}_plain_prealloc", variant, lsym[:2, :33], lidx[:2, :33], lc, ls, lo, fp,
                   False, prealloc=20)
        # alias: cdf_size - 1 = 2^sp (bypass off) and with the escape slot
        # (alias rows hold 2^fp remap entries, so these cases use fp = 12 to stay small)
        sp, afp = 5, 12
        ac, asz = laplace_tables(g, 3, 1 << sp, afp)
        remap, table = ref().rans_alias_build_table(ac, asz, symbol_precision=sp, freq_precision=afp)
        aidx = torch.randint(0, 3, (4, 300), generator=g, dtype=torch.int32)
        asym = sample_from(g, ac, asz, aidx, afp)
        run_coding(f"{variant}_alias", variant, asym, aidx, ac, asz, torch.zeros(3, dtype=torch.int32),
                   afp, False, lookup="alias", push_cdfs=remap, pop_cdfs=table)
        bc, bs, bo = gen_params(g, 2, 15, afp)  # cdf_size 17 -> 16 cuts
        bremap, btable = ref().rans_alias_build_table(bc, bs, symbol_precision=4, freq_precision=afp)
        bsym = torch.randint(-3, 22, (3, 101), generator=g, dtype=torch.int32)
        bidx2 = torch.randint(0, 2, (3, 101), generator=g, dtype=torch.int32)
        run_coding(f"{variant}_alias_bypass", variant, bsym, bidx2, bc, bs, bo, afp, True,
                   lookup="alias", push_cdfs=bremap, pop_cdfs=btable)
        # a cdf that the alias builder rejects (cdf_size - 1 not matching 2^sp cuts): rows stay zero
        rremap, rtable = ref().rans_alias_build_table(bc, bs, symbol_precision=3, freq_precision=afp)
        add(f"{variant}_alias_rejected", meta=np.array(json.dumps(dict(sp=3, fp=afp))), cdfs=bc.numpy(),
            sizes=bs.numpy(), remap=rremap.numpy(), table=rtable.numpy())
        # edge shapes: one symbol, one stream, single-symbol alphabet
        one_c = torch.tensor([[0, 1 << fp]], dtype=torch.int32)
        run_coding(f"{variant}_single_symbol_alphabet", variant, torch.zeros(2, 9, dtype=torch.int32),
                   torch.zeros(2, 9, dtype=torch.int32), one_c, torch.tensor([2], dtype=torch.int32),
                   torch.zeros(1, dtype=torch.int32), fp, False)
        run_coding(f"{variant}_one_symbol", variant, lsym[:1, :1], lidx[:1, :1], lc, ls, lo, fp, False)

    # streaming: two pushes onto one stream, then two partial pops (utils.py:378-393 pattern)
    R = ref()
    for variant in ("rans64", "rans32", "rans32_16"):
        fp = fps[variant]
        cdfs, sizes, offsets = gen_params(g, 3, 20, fp)
        s1 = torch.randint(-2, 24, (3, 50), generator=g, dtype=torch.int32)
        i1 = torch.randint(0, 3, (3, 50), generator=g, dtype=torch.int32)
        s2 = torch.randint(-2, 24, (3, 77), generator=g, dtype=torch.int32)
        i2 = torch.randint(0, 3, (3, 77), generator=g, dtype=torch.int32)
        st = getattr(R, f"{variant}_init_stream")(3)
        push = getattr(R, f"{variant}_push")
        pop = getattr(R, f"{variant}_pop")
        push(st, s2, i2, cdfs, sizes, offsets, freq_precision=fp)
        after1 = st.clone()
        push(st, s1, i1, cdfs, sizes, offsets, freq_precision=fp)
        after2 = st.clone()
        d1 = pop(st, i1, cdfs, sizes, offsets, freq_precision=fp)
        mid = st.clone()
        d2 = pop(st, i2, cdfs, sizes, offsets, freq_precision=fp)
        assert (d1 == s1).all() and (d2 == s2).all()
        add(f"{variant}_streaming", meta=np.array(json.dumps(dict(variant=variant, fp=fp))),
            cdfs=cdfs.numpy(), sizes=sizes.numpy(), offsets=offsets.numpy(), s1=s1.numpy(),
            i1=i1.numpy(), s2=s2.numpy(), i2=i2.numpy(), after1=after1.numpy(), after2=after2.numpy(),
            mid=mid.numpy(), final=st.numpy())

    # table prep known answers
    pm = torch.rand(6, 40, generator=g)
    pm[:, 5:9] = 0.0  # zero-probability symbols -> the borrow repair runs
    pm = pm / pm.sum(-1, keepdim=True)
    out = {}
    for p in (8, 12, 16):
        out[f"cdf{p}"] = R.rans_pmf_to_quantized_cdf(pm, p).numpy()
    add("pmf_to_quantized_cdf", pmf=pm.numpy(), **out)


if __name__ == "__main__":
    main()
    for name, arrays in CASES.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    total = sum(os.path.getsize(os.path.join(HERE, f"{n}.npz")) for n in CASES)
    print(f"wrote {len(CASES)} golden cases, {total / 1024:.1f} KiB")
