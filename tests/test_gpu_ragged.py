"""Ragged coding (rans*_push_ragged / rans*_pop_ragged, tans_push_ragged / tans_pop_ragged) against
the oracle run the way the reference has to run it: one B = 1 call per stream, indexes
arange(n_b), tables = that stream's own rows (the per-element pattern of encode_with_freqs).
Rows must hold identical lengths and payload bytes, pops must return identical symbols."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import golden_cases as G

pytestmark = pytest.mark.gpu

VARIANTS = ["rans64", "rans32", "rans32_16"]


def _per_element_case(rng, variant, bypass, lengths, A=32):
    """One quantised cdf row per symbol (softmax of N(0, 2^2) logits over A symbols)."""
    fp = 15 if variant == "rans32_16" else 16
    T = int(sum(lengths))
    logits = rng.normal(0.0, 2.0, (T, A))
    p = np.exp(logits - logits.max(1, keepdims=True))
    if bypass:
        p = np.concatenate([p, np.full((T, 1), 1e-3 * p.sum(1, keepdims=True).mean())], 1)
    p /= p.sum(1, keepdims=True)
    freqs = np.maximum(1, np.floor(p * ((1 << fp) - p.shape[1])).astype(np.int64)) if T else np.zeros((0, p.shape[1]), np.int64)
    if T:
        freqs[np.arange(T), freqs.argmax(1)] += (1 << fp) - freqs.sum(1)
    cdfs = np.concatenate([np.zeros((T, 1), np.int64), np.cumsum(freqs, 1)], 1).astype(np.int32)
    sizes = np.full(T, cdfs.shape[1], np.int32)
    offs = rng.integers(-4, 4, T).astype(np.int32)
    if bypass:
        sym = rng.integers(-6, A + 6, T).astype(np.int32) + offs
    else:
        u = rng.integers(0, 1 << fp, T)
        sym = (np.array([np.searchsorted(cdfs[i], u[i], side="right") - 1 for i in range(T)], np.int32) + offs)
    return fp, cdfs, sizes, offs, sym.astype(np.int32)


def _oracle_rows(variant, fp, bypass, lengths, sym, cdfs, sizes, offs, idx=None):
    """Per-stream reference calls; returns (pushed rows, popped rows, decoded flat symbols)."""
    pushed, popped, dec = [], [], []
    lo = 0
    for n in lengths:
        hi = lo + int(n)
        init = O.init_stream(variant, 1)
        if n == 0:
            pushed.append(init)
            popped.append(init.copy())
            lo = hi
            continue
        if idx is None:
            tab, ts, to, ix = cdfs[lo:hi], sizes[lo:hi], offs[lo:hi], np.arange(n, dtype=np.int32)[None]
        else:
            tab, ts, to, ix = cdfs, sizes, offs, idx[lo:hi][None]
        st, err = O.push(variant, init, sym[lo:hi][None], ix, tab, ts, to, fp, bypass, 4)
        assert err == 0
        pushed.append(st)
        st2 = st.copy()
        d, derr = O.pop(variant, st2, ix, tab, ts, to, fp, bypass, 4)
        assert derr == 0
        popped.append(st2)
        dec.append(d.reshape(-1))
        lo = hi
    return pushed, popped, (np.concatenate(dec) if dec else np.zeros(0, np.int32))


def _pick_pop(monkeypatch, kernel):
    """"lean": the lean push chain and pop (where the case allows them), "warp" / "thread": the
    general push chain with the general warp-per-stream or thread-per-stream pop."""
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_POP_WARP", "0" if kernel == "thread" else "1")
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_POP_LEAN", "1" if kernel == "lean" else "0")
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_PUSH_LEAN", "1" if kernel == "lean" else "0")


def _same_row(got_row, want):
    return got_row[0] == want[0, 0] and G.payload_bytes(got_row[None]) == G.payload_bytes(want)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("bypass", [False, True])
@pytest.mark.parametrize("pattern", ["per_element", "shared_tables"])
@pytest.mark.parametrize("kernel", ["lean", "warp", "thread"])
def test_ragged_round_trip_matches_per_stream_reference(variant, bypass, pattern, kernel, monkeypatch):
    """Pops through the lean warp kernel (consecutive rows of <= 33 entries without bypass coding;
    other cases fall through to the general one), the general warp-per-stream kernel (rows of <= 64
    entries) and the thread-per-stream kernel."""
    from torch_ans_b200 import _C
    _pick_pop(monkeypatch, kernel)
    rng = np.random.default_rng(zlib.crc32(f"ragged-{variant}-{bypass}-{pattern}".encode()))
    lengths = [0, 1, 3, 4, 5, 17, 64, 257, 1000, 2] + list(rng.integers(0, 400, 30))
    fp, cdfs, sizes, offs, sym = _per_element_case(rng, variant, bypass, lengths)
    idx = None
    if pattern == "shared_tables":  # a few shared rows, explicit indexes per symbol
        K = 7
        cdfs, sizes, offs = cdfs[:K].copy(), sizes[:K].copy(), offs[:K].copy()
        idx = rng.integers(0, K, len(sym)).astype(np.int32)
        if not bypass:  # resample symbols from their table
            u = rng.integers(0, 1 << fp, len(sym))
            sym = np.array([np.searchsorted(cdfs[k], x, side="right") - 1 for k, x in zip(idx, u)], np.int32) + offs[idx]
        else:
            sym = (rng.integers(-6, cdfs.shape[1] + 4, len(sym)) + offs[idx]).astype(np.int32)
    pushed, popped, dec_ref = _oracle_rows(variant, fp, bypass, lengths, sym, cdfs, sizes, offs, idx)
    rows = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int64)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    B = len(lengths)
    st = getattr(_C, f"{variant}_init_stream")(B).cuda()
    kw = dict(freq_precision=fp, bypass_coding=bypass, bypass_precision=4)
    getattr(_C, f"{variant}_push_ragged")(st, dev(sym), rows.cuda(), dev(cdfs), dev(sizes),
                                          indexes=None if idx is None else dev(idx), offsets=dev(offs), **kw)
    assert _C.device_status() == 0
    got = st.cpu().numpy()
    for b in range(B):
        assert _same_row(got[b], pushed[b]), f"stream {b} (length {lengths[b]})"
    dec = getattr(_C, f"{variant}_pop_ragged")(st, rows, dev(cdfs), dev(sizes),
                                               indexes=None if idx is None else dev(idx), offsets=dev(offs), **kw)
    assert _C.device_status() == 0
    assert np.array_equal(dec.cpu().numpy(), dec_ref) and np.array_equal(dec_ref, sym)
    got = st.cpu().numpy()
    for b in range(B):
        assert _same_row(got[b], popped[b]), f"stream {b} after pop"


@pytest.mark.parametrize("variant", VARIANTS)
def test_ragged_bad_rows_and_indexes_are_flagged(variant):
    """An index past the table list skips its step with TANS_DEV_BAD_INDEX (as the rectangular ops
    do); a row whose range lies outside the flat arrays is left untouched with TANS_DEV_BAD_VALUE;
    the other rows are still coded exactly."""
    from torch_ans_b200 import _C
    rng = np.random.default_rng(7)
    fp, cdfs, sizes, offs, sym = _per_element_case(rng, variant, False, [5, 6, 7])
    T = len(sym)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    kw = dict(freq_precision=fp, bypass_coding=False)
    # bad index in stream 1 (symbol 7): the oracle restatement skips that step the same way
    idx = np.arange(T, dtype=np.int32)
    idx[7] = T + 5
    rows = torch.tensor([0, 5, 11, 18], dtype=torch.int64)
    st = getattr(_C, f"{variant}_init_stream")(3).cuda()
    getattr(_C, f"{variant}_push_ragged")(st, dev(sym), rows.cuda(), dev(cdfs), dev(sizes), indexes=dev(idx),
                                          offsets=dev(offs), **kw)
    assert _C.device_status() == O.ERR_BAD_INDEX
    want, err = O.push(variant, O.init_stream(variant, 1), sym[5:11][None], idx[5:11][None], cdfs, sizes, offs, fp,
                       False)
    assert err == O.ERR_BAD_INDEX
    assert _same_row(st.cpu().numpy()[1], want)
    # invalid ranges: stream 1 runs past the arrays, stream 2 ends before it starts
    bad = torch.tensor([0, 5, 30, 18], dtype=torch.int64).cuda()
    st = getattr(_C, f"{variant}_init_stream")(3).cuda()
    init = st.cpu().numpy().copy()
    getattr(_C, f"{variant}_push_ragged")(st, dev(sym), bad, dev(cdfs), dev(sizes), offsets=dev(offs), **kw)
    assert _C.device_status() == O.ERR_BAD_VALUE
    got = st.cpu().numpy()
    want0, _ = O.push(variant, O.init_stream(variant, 1), sym[0:5][None], np.arange(5, dtype=np.int32)[None],
                      cdfs[0:5], sizes[0:5], offs[0:5], fp, False)
    assert _same_row(got[0], want0)
    assert np.array_equal(got[1, :init.shape[1]], init[1]) and np.array_equal(got[2, :init.shape[1]], init[2])


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("case", ["unsorted_rows", "wide_rows", "short_table", "narrow_rows"])
@pytest.mark.parametrize("kernel", ["lean", "warp"])
def test_ragged_pop_unusual_rows(variant, case, kernel, monkeypatch):
    """Rows the ballot search must not take (entries out of order: the reference bisection's
    answer then differs from a count unless the comparison mask is still a prefix, so the kernel
    runs the bisection itself), rows wider than 64 entries (the thread-per-stream kernel), a
    per-element table list shorter than the symbols (the steps past it are bad indexes) and rows
    of 21 entries (fewer than the lanes).  Decoded symbols, rows and error bits must match the
    oracle's per-stream pops of the same streams."""
    from torch_ans_b200 import _C
    _pick_pop(monkeypatch, kernel)
    rng = np.random.default_rng(zlib.crc32(f"unusual-{variant}-{case}".encode()))
    lengths = [0, 1, 9, 40, 33, 70, 3]
    A = {"wide_rows": 100, "narrow_rows": 20}.get(case, 32)
    fp, cdfs, sizes, offs, sym = _per_element_case(rng, variant, False, lengths, A=A)
    pushed, _, _ = _oracle_rows(variant, fp, False, lengths, sym, cdfs, sizes, offs)
    pop_cdfs = cdfs.copy()
    if case == "unsorted_rows":  # swap two interior entries of every third row after the push
        for i in range(0, len(sym), 3):
            a, b = 5 + i % 7, 20 + i % 9
            pop_cdfs[i, a], pop_cdfs[i, b] = pop_cdfs[i, b], pop_cdfs[i, a]
    if case == "short_table":  # the last 50 symbols have no row
        pop_cdfs, sizes, offs = pop_cdfs[:-50].copy(), sizes[:-50].copy(), offs[:-50].copy()
    # oracle pops of each stream with the (possibly unsorted) rows; symbol i of the batch reads row i
    dec_ref, rows_ref, err_ref = [], [], 0
    lo = 0
    for b, n in enumerate(lengths):
        st = pushed[b].copy()
        if n:
            d, e = O.pop(variant, st, np.arange(lo, lo + n, dtype=np.int32)[None], pop_cdfs, sizes, offs, fp,
                         False)
            dec_ref.append(d.reshape(-1))
            err_ref |= e
        rows_ref.append(st)
        lo += n
    dec_ref = np.concatenate(dec_ref)
    Wd = max(r.shape[1] for r in pushed)
    host = np.zeros((len(lengths), Wd), np.int32)
    for b, r in enumerate(pushed):
        host[b, : r.shape[1]] = r[0]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = dev(host)
    rows = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int64)
    dec = getattr(_C, f"{variant}_pop_ragged")(st, rows, dev(pop_cdfs), dev(sizes), offsets=dev(offs),
                                               freq_precision=fp, bypass_coding=False)
    assert _C.device_status() == err_ref
    assert np.array_equal(dec.cpu().numpy(), dec_ref)
    got = st.cpu().numpy()
    for b in range(len(lengths)):
        assert _same_row(got[b], rows_ref[b]), f"stream {b}"


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("kernel", ["lean", "warp", "thread"])
def test_ragged_pop_past_the_pushed_words(variant, kernel, monkeypatch):
    """Each stream pops a few more symbols than were pushed into it: the extra steps read below
    the first data word (TANS_DEV_UNDERFLOW, zero words, as the oracle's per-stream pops do) and the
    decoded symbols, the rows left behind (state and length, which goes negative) and the error
    bits must still equal the oracle's."""
    from torch_ans_b200 import _C
    _pick_pop(monkeypatch, kernel)
    rng = np.random.default_rng(zlib.crc32(f"past-{variant}".encode()))
    pushed_n = [0, 1, 2, 7, 31, 64, 100, 5]
    extra = [3, 1, 6, 9, 2, 40, 5, 17]
    pop_n = [a + e for a, e in zip(pushed_n, extra)]
    fp, cdfs, sizes, offs, sym = _per_element_case(rng, variant, False, pop_n)
    starts = np.concatenate([[0], np.cumsum(pop_n)])
    dec_ref, rows_ref, err_ref = [], [], 0
    for b, (n, m) in enumerate(zip(pushed_n, pop_n)):
        lo = int(starts[b])
        st = O.init_stream(variant, 1)
        if n:
            st, e = O.push(variant, st, sym[lo:lo + n][None], np.arange(n, dtype=np.int32)[None],
                           cdfs[lo:lo + n], sizes[lo:lo + n], offs[lo:lo + n], fp, False)
            assert e == 0
        rows_ref.append(st.copy())
        d, e = O.pop(variant, st, np.arange(m, dtype=np.int32)[None], cdfs[lo:lo + m], sizes[lo:lo + m],
                     offs[lo:lo + m], fp, False)
        assert np.array_equal(d.reshape(-1)[:n], sym[lo:lo + n])
        dec_ref.append(d.reshape(-1))
        err_ref |= e
        rows_ref[-1] = (rows_ref[-1], st)
    assert err_ref & O.ERR_UNDERFLOW
    Wd = max(r[0].shape[1] for r in rows_ref)
    host = np.zeros((len(pop_n), Wd), np.int32)
    for b, (r, _) in enumerate(rows_ref):
        host[b, : r.shape[1]] = r[0]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = dev(host)
    dec = getattr(_C, f"{variant}_pop_ragged")(st, torch.from_numpy(starts.astype(np.int64)), dev(cdfs), dev(sizes),
                                               offsets=dev(offs), freq_precision=fp, bypass_coding=False)
    assert _C.device_status() == err_ref
    assert np.array_equal(dec.cpu().numpy(), np.concatenate(dec_ref))
    got = st.cpu().numpy()
    head = 3 if variant == "rans64" else 2  # the length word and the state
    for b, (_, want) in enumerate(rows_ref):
        assert np.array_equal(got[b][:head], want[0, :head]), f"stream {b}"


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("kernel", ["lean", "warp"])
def test_ragged_push_steps_wider_than_the_precision(variant, kernel, monkeypatch):
    """Per-element rows with a start of -2^30 and a step of 2^24 - 1 (far above 2^fp): the
    reference still codes them and its 32-bit states then leave [0, 2^31), where only the exact
    step code divides correctly.  Rows must equal the oracle's per-stream pushes."""
    from torch_ans_b200 import _C
    from tests.test_gpu_parity import wide_step_case
    _pick_pop(monkeypatch, kernel)
    rng = np.random.default_rng(zlib.crc32(f"ragged-wide-{variant}".encode()))
    lengths = [0, 3, 400, 17, 256, 99]
    fp, tabs, tsizes, toffs, sym2, idx2 = wide_step_case(rng, 1, int(sum(lengths)))
    sym, k = sym2.reshape(-1), idx2.reshape(-1)
    cdfs, sizes, offs = tabs[k], tsizes[k], toffs[k]  # one row per symbol
    pushed, _, _ = _oracle_rows_push_only(variant, fp, lengths, sym, cdfs, sizes, offs)
    rows = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int64)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    st = getattr(_C, f"{variant}_init_stream")(len(lengths)).cuda()
    getattr(_C, f"{variant}_push_ragged")(st, dev(sym), rows.cuda(), dev(cdfs), dev(sizes), offsets=dev(offs),
                                          freq_precision=fp, bypass_coding=False)
    assert _C.device_status() == 0
    got = st.cpu().numpy()
    for b in range(len(lengths)):
        assert _same_row(got[b], pushed[b]), f"stream {b} (length {lengths[b]})"


def _oracle_rows_push_only(variant, fp, lengths, sym, cdfs, sizes, offs):
    pushed, lo = [], 0
    for n in lengths:
        hi = lo + int(n)
        st = O.init_stream(variant, 1)
        if n:
            st, err = O.push(variant, st, sym[lo:hi][None], np.arange(n, dtype=np.int32)[None], cdfs[lo:hi],
                             sizes[lo:hi], offs[lo:hi], fp, False)
            assert err == 0
        pushed.append(st)
        lo = hi
    return pushed, None, None


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("kernel", ["lean", "warp"])
def test_ragged_push_rows_too_short(variant, kernel, monkeypatch):
    """Rows sized by the caller too short for their words (the C ABI): every push chain keeps the
    words that fit, counts the rest in the length, flags TANS_DEV_OVERFLOW and never writes past
    the row (guard words after the last row, and each row's neighbour, stay intact), exactly as the
    oracle's per-stream pushes into rows of the same width do."""
    from torch_ans_b200 import capi
    _pick_pop(monkeypatch, kernel)
    lib = capi.load()
    rng = np.random.default_rng(zlib.crc32(f"ragged-ovf-{variant}".encode()))
    lengths = [0, 2, 40, 300, 7, 120, 64]
    fp, cdfs, sizes, offs, sym = _per_element_case(rng, variant, False, lengths)
    B = len(lengths)
    init = O.init_stream(variant, 1)
    W = init.shape[1] + 5  # room for a few words only
    host = np.zeros((B, W), np.int32)
    host[:, : init.shape[1]] = init[0]
    want, err_ref = [], 0
    lo = 0
    for n in lengths:
        row = host[:1].copy()
        if n:
            e = O.lib().orc_push(O.VARIANTS[variant], 0, 1, O._ptr(row), 1, W, O._ptr(np.ascontiguousarray(sym[lo:lo + n])),
                                 O._ptr(np.arange(n, dtype=np.int32)), n, O._ptr(np.ascontiguousarray(cdfs[lo:lo + n])),
                                 n, cdfs.shape[1], O._ptr(np.ascontiguousarray(sizes[lo:lo + n])),
                                 O._ptr(np.ascontiguousarray(offs[lo:lo + n])), fp, 0, 4, 1)
            err_ref |= int(e)
        want.append(row[0])
        lo += n
    assert err_ref & O.ERR_OVERFLOW
    guard = 8
    flat = torch.full((B * W + guard,), 0x5A5A5A5A, dtype=torch.int32, device="cuda")
    flat[: B * W] = torch.from_numpy(host).cuda().reshape(-1)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    s_d, c_d, z_d, o_d = dev(sym), dev(cdfs), dev(sizes), dev(offs)
    rows = dev(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64))
    T = len(sym)
    ws = torch.empty(lib.tans_push_ragged_workspace_size(T) + 256, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    cs = torch.cuda.current_stream().cuda_stream
    rc = lib.tans_push_ragged(capi.VARIANT[variant], flat.data_ptr(), B, W, s_d.data_ptr(), None, rows.data_ptr(), T,
                              c_d.data_ptr(), T, cdfs.shape[1], z_d.data_ptr(), o_d.data_ptr(), fp, 0, 4,
                              ws.data_ptr(), ws.numel(), status.data_ptr(), cs)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == err_ref
    got = flat.cpu().numpy()
    assert (got[B * W:] == 0x5A5A5A5A).all()
    for b in range(B):
        assert np.array_equal(got[b * W:(b + 1) * W], want[b]), f"stream {b} (length {lengths[b]})"
