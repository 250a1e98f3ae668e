"""GPU parity tests: the CUDA coding path against the reference's golden vectors and the oracle.

Bar: bit-exact.  Every pushed stream must have the reference's row width, length column and
payload bytes; every pop must return the identical int32 symbols and leave the identical row
length and state.  Paths covered: the `_C` op surface (what the reference's callers bind) and the
raw C ABI through ctypes (what a non-torch host binds).
"""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import golden_cases as G

pytestmark = pytest.mark.gpu

VARIANTS = ["rans64", "rans32", "rans32_16"]
FP = {"rans64": 16, "rans32": 16, "rans32_16": 15}


@pytest.fixture(scope="module")
def C():
    from torch_ans_b200 import _C
    _C.set_sync_check(False)
    _C.device_status(reset=True)
    return _C


def op_names(variant, interleave, alias_push, lookup):
    if interleave == 4:
        push = f"{variant}_i4_push"
        pop = f"{variant}_i4_invcdf_pop" if lookup == "invcdf" else f"{variant}_i4_pop"
    else:
        push = f"{variant}_alias_push" if alias_push else f"{variant}_push"
        pop = {"alias": f"{variant}_alias_pop", "invcdf": f"{variant}_invcdf_pop", "search": f"{variant}_pop"}[lookup]
    return push, pop


def same_rows(a, b):
    """Equal shapes, lengths and records (state and words up to each row's length).  Columns that a
    resize added past the old width are left uninitialised by the reference (rans.hpp:120-122:
    `resize_` then the old rows copied back), so past the length only the rows' old width is
    defined; test_push_onto_popped_stream_keeps_old_words compares that region too."""
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a[:, 0], b[:, 0]) and G.payload_bytes(a) == G.payload_bytes(b)


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name", G.coding_cases())
def test_golden_through_op_surface(C, name):
    d = G.load(name)
    m = d["meta"]
    push, pop = op_names(m["variant"], m["interleave"], m["alias_push"], m["lookup"])
    kw = dict(freq_precision=m["fp"], bypass_coding=bool(m["bypass"]), bypass_precision=m["bp"])
    stream = t(d["stream_in"])
    getattr(C, push)(stream, t(d["symbols"]), t(d["indexes"]), t(d["push_cdfs"]), t(d["sizes"]), t(d["offsets"]), **kw)
    assert C.device_status() == 0
    got = stream.cpu().numpy()
    assert got.shape == d["pushed"].shape
    assert np.array_equal(got[:, 0], d["pushed"][:, 0])
    assert G.payload_bytes(got) == d["pushed_bytes"].tobytes()
    assert b"".join(C.rans_stream_to_byte_strings(stream)) == d["pushed_bytes"].tobytes()
    st2 = C.rans_byte_strings_to_stream(C.rans_stream_to_byte_strings(stream)).cuda()
    dec = getattr(C, pop)(st2, t(d["indexes"]), t(d["pop_cdfs"]), t(d["sizes"]), t(d["offsets"]), **kw)
    assert C.device_status() == 0
    assert np.array_equal(dec.cpu().numpy(), d["decoded"])
    assert same_rows(st2.cpu().numpy(), d["popped"])


@pytest.mark.parametrize("name", [n for n in G.coding_cases() if "i4" not in n][::2])
def test_golden_through_c_abi(name):
    """Same golden cases, calling libtorch_ans_b200 directly with device pointers (ctypes)."""
    from torch_ans_b200 import capi
    lib = capi.load()
    d = G.load(name)
    m = d["meta"]
    v = capi.VARIANT[m["variant"]]
    W = O.resized_width(d["stream_in"], d["symbols"].shape[1], m["fp"], bool(m["bypass"]))
    host = np.zeros((d["stream_in"].shape[0], W), np.int32)
    host[:, : d["stream_in"].shape[1]] = d["stream_in"]
    stream = t(host)
    sym, idx, pc, sz, off = t(d["symbols"]), t(d["indexes"]), t(d["push_cdfs"]), t(d["sizes"]), t(d["offsets"])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    cs = torch.cuda.current_stream().cuda_stream
    B, N = sym.shape
    K, Wc = pc.shape
    ws_bytes = lib.tans_push_workspace_size(v, K, Wc)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device="cuda")
    rc = lib.tans_push(v, int(m["alias_push"]), 1, stream.data_ptr(), B, W, sym.data_ptr(), idx.data_ptr(), N,
                       pc.data_ptr(), K, Wc, sz.data_ptr(), off.data_ptr(), m["fp"], m["bypass"], m["bp"],
                       ws.data_ptr(), ws.numel(), status.data_ptr(), cs)
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    got = stream.cpu().numpy()
    assert np.array_equal(got[:, 0], d["pushed"][:, 0]) and G.payload_bytes(got) == d["pushed_bytes"].tobytes()
    # pop with the library allocating its own scratch (workspace = NULL)
    qc = t(d["pop_cdfs"])
    out = torch.empty_like(idx)
    rc = lib.tans_pop(v, capi.LOOKUP[m["lookup"]], 1, stream.data_ptr(), B, W, out.data_ptr(), idx.data_ptr(), N,
                      qc.data_ptr(), qc.shape[0], qc.shape[1], sz.data_ptr(), off.data_ptr(), m["fp"], m["bypass"],
                      m["bp"], None, 0, status.data_ptr(), cs)
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    assert np.array_equal(out.cpu().numpy(), d["decoded"])
    got = stream.cpu().numpy()  # popped in place on the push-width row: compare lengths and payload
    assert np.array_equal(got[:, 0], d["popped"][:, 0]) and G.payload_bytes(got) == G.payload_bytes(d["popped"])


@pytest.mark.parametrize("variant", VARIANTS)
def test_streaming_pushes_and_partial_pops(C, variant):
    d = G.load(f"{variant}_streaming")
    fp = d["meta"]["fp"]
    cdfs, sizes, offs = t(d["cdfs"]), t(d["sizes"]), t(d["offsets"])
    st = getattr(C, f"{variant}_init_stream")(3).cuda()
    push, pop = getattr(C, f"{variant}_push"), getattr(C, f"{variant}_pop")
    push(st, t(d["s2"]), t(d["i2"]), cdfs, sizes, offs, freq_precision=fp)
    assert same_rows(st.cpu().numpy(), d["after1"])
    push(st, t(d["s1"]), t(d["i1"]), cdfs, sizes, offs, freq_precision=fp)
    assert same_rows(st.cpu().numpy(), d["after2"])
    d1 = pop(st, t(d["i1"]), cdfs, sizes, offs, freq_precision=fp)
    assert np.array_equal(d1.cpu().numpy(), d["s1"]) and same_rows(st.cpu().numpy(), d["mid"])
    d2 = pop(st, t(d["i2"]), cdfs, sizes, offs, freq_precision=fp)
    assert np.array_equal(d2.cpu().numpy(), d["s2"]) and same_rows(st.cpu().numpy(), d["final"])
    assert C.device_status() == 0


def _random_case(rng, variant, bypass, K=5, A=40, fp=None):
    fp = FP[variant] if fp is None else fp
    pm = rng.integers(1, 1024, (K, A)).astype(np.float32)
    pm = np.concatenate([pm, np.ones((K, 1), np.float32)], 1)
    pm /= pm.sum(1, keepdims=True)
    cdfs = O.pmf_to_quantized_cdf(pm, fp)
    sizes = np.full(K, A + 2, np.int32)
    offs = rng.integers(-8, 8, K).astype(np.int32)
    return fp, cdfs, sizes, offs


def _random_combos():
    """Every op the reference has (no 4-state alias op, no rans64_i4_invcdf_pop) through every
    table path that applies (4-state pops read the caller's tables directly in every mode)."""
    out = []
    for table_path in ("fused", "direct", "fused_small"):
        for lookup in ("search", "invcdf", "alias"):
            for interleave in (1, 4):
                for bypass in (False, True):
                    for variant in VARIANTS:
                        if interleave == 4 and (lookup == "alias" or table_path != "fused" or
                                                (lookup == "invcdf" and variant == "rans64")):
                            continue
                        out.append(pytest.param(variant, bypass, interleave, lookup, table_path,
                                                id=f"{table_path}-{lookup}-{interleave}-{bypass}-{variant}"))
    return out


@pytest.mark.parametrize("variant,bypass,interleave,lookup,table_path", _random_combos())
def test_random_against_oracle(C, variant, bypass, interleave, lookup, table_path, monkeypatch):
    """Seeded cases with odd lengths and misaligned rows (vector and scalar load paths), through
    each decode table path: fused table in L2 ("fused"), fused table small enough for shared
    memory ("fused_small", fp 11), and the caller's tables read directly ("direct")."""
    monkeypatch.setenv("TORCH_ANS_B200_FUSED", "0" if table_path == "direct" else "1")
    rng = np.random.default_rng(zlib.crc32(f"{variant}-{bypass}-{interleave}-{lookup}-{table_path}".encode()))
    if lookup == "alias":
        fp = 12
        K, sp = 3, 5
        A = 1 << sp  # cdf_size - 1 must equal the 2^sp alias cuts; with escapes the last slot is the escape
        pm = rng.random((K, A)) + 0.05
        cdfs = O.pmf_to_quantized_cdf((pm / pm.sum(1, keepdims=True)).astype(np.float32), fp)
        sizes = np.full(K, A + 1, np.int32)
        offs = rng.integers(-3, 3, K).astype(np.int32)
        push_c, pop_c, ok = O.alias_build_table(cdfs, sizes, sp, fp)
        assert ok == K
        lo, hi = (-5, A + 5) if bypass else (0, A)
    else:
        fp, cdfs, sizes, offs = _random_case(rng, variant, bypass, fp=11 if table_path == "fused_small" else None)
        push_c = cdfs
        pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
        A = cdfs.shape[1] - 2
        lo, hi = (-20, A + 20) if bypass else (0, A + 1)
    K = cdfs.shape[0]
    B, N = 37, 1001
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = (rng.integers(lo, hi, (B, N)) + (offs[idx] if not bypass else 0)).astype(np.int32)
    if not bypass:
        sym = np.clip(sym - offs[idx], 0, sizes[idx] - 2) + offs[idx]
        sym = sym.astype(np.int32)
    ref_stream, perr = O.push(variant, O.init_stream(variant, B, interleave), sym, idx, push_c, sizes, offs, fp, bypass,
                              4, alias=(lookup == "alias"), interleave=interleave)
    assert perr == 0
    ref_pop_stream = ref_stream.copy()
    ref_dec, derr = O.pop(variant, ref_pop_stream, idx, pop_c, sizes, offs, fp, bypass, 4, lookup=lookup,
                          interleave=interleave)
    assert derr == 0 and np.array_equal(ref_dec, sym)
    push, pop = op_names(variant, interleave, lookup == "alias", lookup)
    # misaligned inputs: views one element into bigger buffers force the scalar load path
    for misalign in (0, 1):
        big_s = torch.zeros(B * N + 1, dtype=torch.int32, device="cuda")
        big_i = torch.zeros(B * N + 1, dtype=torch.int32, device="cuda")
        big_s[misalign:misalign + B * N] = t(sym).reshape(-1)
        big_i[misalign:misalign + B * N] = t(idx).reshape(-1)
        s_in = big_s[misalign:misalign + B * N].view(B, N)
        i_in = big_i[misalign:misalign + B * N].view(B, N)
        st = getattr(C, f"{variant}_init_stream")(B, interleave).cuda()
        kw = dict(freq_precision=fp, bypass_coding=bypass, bypass_precision=4)
        getattr(C, push)(st, s_in, i_in, t(push_c), t(sizes), t(offs), **kw)
        assert C.device_status() == 0
        assert same_rows(st.cpu().numpy(), ref_stream)
        dec = getattr(C, pop)(st, i_in, t(pop_c), t(sizes), t(offs), **kw)
        assert C.device_status() == 0
        assert np.array_equal(dec.cpu().numpy(), sym)
        assert same_rows(st.cpu().numpy(), ref_pop_stream)


@pytest.mark.parametrize("variant", VARIANTS)
def test_error_bits_match_oracle(C, variant):
    """Invalid table indexes and out-of-range symbols are flagged, not read out of bounds."""
    fp = FP[variant]
    cdfs = np.array([[0, 10, 20, 1 << fp]], np.int32)
    sizes = np.array([4], np.int32)
    sym = np.array([[0, 5, 1, 2, 0]], np.int32)
    idx = np.array([[0, 0, 3, 0, -1]], np.int32)
    ref, err = O.push(variant, O.init_stream(variant, 1), sym, idx, cdfs, sizes, None, fp, False)
    st = getattr(C, f"{variant}_init_stream")(1).cuda()
    getattr(C, f"{variant}_push")(st, t(sym), t(idx), t(cdfs), t(sizes), freq_precision=fp, bypass_coding=False)
    bits = C.device_status()
    assert bits == err and bits & O.ERR_BAD_INDEX and bits & O.ERR_BAD_VALUE
    assert same_rows(st.cpu().numpy(), ref)
    C.set_sync_check(True)
    try:
        with pytest.raises(RuntimeError, match="table-index-out-of-range"):
            getattr(C, f"{variant}_push")(st, t(sym), t(idx), t(cdfs), t(sizes), freq_precision=fp, bypass_coding=False)
    finally:
        C.set_sync_check(False)
    C.device_status()


def test_pmf_to_quantized_cdf_on_gpu_matches_reference(C):
    d = G.load("pmf_to_quantized_cdf")
    for p in (8, 12, 16):
        got = C.rans_pmf_to_quantized_cdf(t(d["pmf"]), p)
        assert got.is_cuda and np.array_equal(got.cpu().numpy(), d[f"cdf{p}"])
    assert C.rans_pmf_to_quantized_cdf(torch.tensor([0.25] * 4).cuda(), 8).tolist() == [0, 64, 128, 192, 256]
    assert C.rans_pmf_to_quantized_cdf(torch.tensor([0.1, 0.2, 0.3, 0.4]).cuda(), 8).tolist() == [0, 26, 77, 154, 256]
    # a CPU pmf is computed on the GPU and returned on the CPU
    assert C.rans_pmf_to_quantized_cdf(torch.tensor([0.1, 0.2, 0.3, 0.4]), 8).device.type == "cpu"


def test_device_stream_helpers():
    from torch_ans_b200 import capi
    lib = capi.load()
    cs = torch.cuda.current_stream().cuda_stream
    for variant, ilv in (("rans64", 1), ("rans32", 4), ("rans32_16", 4)):
        W = 1 + ilv * (8 if variant == "rans64" else 4) // 4 + 5
        s = torch.full((6, W), 7, dtype=torch.int32, device="cuda")
        assert lib.tans_init_stream(capi.VARIANT[variant], ilv, s.data_ptr(), 6, W, cs) == 0
        ref = np.zeros((6, W), np.int32)
        ref[:, : O.init_stream(variant, 6, ilv).shape[1]] = O.init_stream(variant, 6, ilv)
        assert np.array_equal(s.cpu().numpy(), ref)
    d = G.load("rans32_bypass")
    st = t(d["pushed"])
    segs = O.stream_to_byte_strings(d["pushed"])
    mx = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.tans_stream_max_length(st.data_ptr(), st.shape[0], st.shape[1], mx.data_ptr(), cs) == 0
    assert mx.item() == max(len(x) for x in segs)
    from torch_ans_b200 import _C
    for nb in (1, 2, 4, 8):
        for ns in (None, len(segs)):
            if nb == 1 and max(len(x) for x in segs) > 255:
                # the reference's struct.pack("B", n) raises for n > 255; so does the device path
                with pytest.raises(ValueError):
                    _C.stream_to_merged_bytes(st, nb, ns)
                continue
            assert _C.stream_to_merged_bytes(st, nb, ns) == O.merge_bytes(segs, nb, ns)
            packed = _C.stream_to_merged_tensor(st, nb, ns)
            assert bytes(packed.cpu().numpy().tobytes()) == O.merge_bytes(segs, nb, ns)
            if nb != 8:
                back = _C.merged_tensor_to_stream(packed.cpu(), nb, ns, "cuda")
                assert same_rows(back.cpu().numpy(), O.byte_strings_to_stream(segs))
    # scatter back
    lens = torch.tensor([len(x) for x in segs], dtype=torch.int32, device="cuda")
    offs = torch.tensor(np.concatenate([[0], np.cumsum([len(x) for x in segs])[:-1]]), dtype=torch.int64, device="cuda")
    flat = torch.tensor(np.frombuffer(b"".join(segs), np.uint8).copy(), device="cuda")
    out = torch.full_like(st, -1)
    assert lib.tans_scatter_payloads(flat.data_ptr(), offs.data_ptr(), lens.data_ptr(), out.data_ptr(), st.shape[0],
                                     st.shape[1], cs) == 0
    assert same_rows(out.cpu().numpy(), d["pushed"])


LAYOUTS = ["fused_smem", "split_smem", "fused_global", "split_global", "bucket_global", "generic"]


def _layout_combos():
    """Layouts a lookup can use (alias offsets depend on cum: fused layouts only; fused_global
    serves alias tables when several streams share a thread), streams per thread only for the
    fast kernel (the lean one runs one stream per thread)."""
    out = []
    for kernel in ("lean", "fast"):
        for spt in ("1", "4"):
            for bypass in (False, True):
                for lookup in ("search", "invcdf", "alias"):
                    for variant in VARIANTS:
                        for layout in LAYOUTS:
                            if layout in ("split_smem", "split_global", "bucket_global") and lookup == "alias":
                                continue
                            if layout == "fused_global" and lookup != "alias" and spt == "4":
                                continue
                            if kernel == "lean" and spt == "4":
                                continue
                            out.append(pytest.param(layout, variant, lookup, bypass, spt, kernel,
                                                    id=f"{kernel}-{spt}-{bypass}-{lookup}-{variant}-{layout}"))
    return out


@pytest.mark.parametrize("layout,variant,lookup,bypass,spt,kernel", _layout_combos())
def test_fast_pop_layouts(C, layout, variant, lookup, bypass, spt, kernel, monkeypatch):
    """Aligned rows with a length divisible by 4 take the lean pop kernel (one stream per thread,
    shortest serial step) or the fast one (several streams per thread); every table layout they
    can use is forced in turn (an infeasible one falls back to the automatic choice) and must
    decode exactly what the oracle decodes, with the same final stream rows."""
    monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", kernel)
    monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", layout)
    monkeypatch.setenv("TORCH_ANS_B200_SPT", spt)
    rng = np.random.default_rng(zlib.crc32(f"fast-{layout}-{variant}-{lookup}-{bypass}-{spt}".encode()))
    if lookup == "alias":
        fp, K, sp = 12, 3, 5
        A = 1 << sp
        pm = rng.random((K, A)) + 0.05
        cdfs = O.pmf_to_quantized_cdf((pm / pm.sum(1, keepdims=True)).astype(np.float32), fp)
        sizes = np.full(K, A + 1, np.int32)
        offs = rng.integers(-3, 3, K).astype(np.int32)
        push_c, pop_c, ok = O.alias_build_table(cdfs, sizes, sp, fp)
        lo, hi = (-5, A + 5) if bypass else (0, A)
    else:
        fp = 11 if layout.endswith("smem") else FP[variant]
        fp, cdfs, sizes, offs = _random_case(rng, variant, bypass, K=4, A=30, fp=fp)
        push_c = cdfs
        pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
        A = cdfs.shape[1] - 2
        lo, hi = (-20, A + 20) if bypass else (0, A + 1)
    K = cdfs.shape[0]
    B, N = 45, 1000
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = rng.integers(lo, hi, (B, N)).astype(np.int32)
    if not bypass:
        sym = (np.clip(sym, 0, sizes[idx] - 2) + offs[idx]).astype(np.int32)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, push_c, sizes, offs, fp, bypass, 4,
                       alias=lookup == "alias")
    assert perr == 0
    ref_pop = ref.copy()
    dec_ref, derr = O.pop(variant, ref_pop, idx, pop_c, sizes, offs, fp, bypass, 4, lookup=lookup)
    assert derr == 0 and np.array_equal(dec_ref, sym)
    push, pop = op_names(variant, 1, lookup == "alias", lookup)
    kw = dict(freq_precision=fp, bypass_coding=bypass, bypass_precision=4)
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, push)(st, t(sym), t(idx), t(push_c), t(sizes), t(offs), **kw)
    assert same_rows(st.cpu().numpy(), ref)
    dec = getattr(C, pop)(st, t(idx), t(pop_c), t(sizes), t(offs), **kw)
    assert C.device_status() == 0
    assert np.array_equal(dec.cpu().numpy(), sym)
    assert same_rows(st.cpu().numpy(), ref_pop)


PUSH_KERNELS = ["ws", "chunk", "generic"]


def _push_case(rng, variant, alias, bypass, B, N):
    """Tables and symbols for a push-kernel test: random cdfs (with escapes when `bypass`), or
    alias remap rows."""
    if alias:
        fp, K, sp = 12, 3, 5
        A = 1 << sp
        pm = rng.random((K, A)) + 0.05
        cdfs = O.pmf_to_quantized_cdf((pm / pm.sum(1, keepdims=True)).astype(np.float32), fp)
        sizes = np.full(K, A + 1, np.int32)
        offs = rng.integers(-3, 3, K).astype(np.int32)
        push_c, _, ok = O.alias_build_table(cdfs, sizes, sp, fp)
        assert ok == K
        lo, hi = (-5, A + 5) if bypass else (0, A)
    else:
        fp, cdfs, sizes, offs = _random_case(rng, variant, bypass, K=6, A=30)
        push_c = cdfs
        A = cdfs.shape[1] - 2
        lo, hi = (-20, A + 20) if bypass else (0, A + 1)
    K = cdfs.shape[0]
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = rng.integers(lo, hi, (B, N)).astype(np.int32)
    if not bypass:
        sym = (np.clip(sym, 0, sizes[idx] - 2) + offs[idx]).astype(np.int32)
    return fp, push_c, sizes, offs, sym, idx


@pytest.mark.parametrize("kernel", PUSH_KERNELS)
@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("alias", [False, True])
@pytest.mark.parametrize("bypass", [False, True])
@pytest.mark.parametrize("shape", [(3, 4), (45, 1000), (700, 252)])
def test_fast_push_kernels(C, kernel, variant, alias, bypass, shape, monkeypatch):
    """Aligned rows with a length divisible by 4 take a fast push kernel: the warp-specialised one
    ("ws": chain warps fed by prep warps through a shared-memory ring), the single-role one
    ("chunk") or the generic one, forced in turn.  Each must write exactly the oracle's rows
    (length, state, words), with stream counts that leave blocks and warps partly filled and
    lengths that leave the last group of chunks partial."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", kernel)
    B, N = shape
    rng = np.random.default_rng(zlib.crc32(f"pushk-{kernel}-{variant}-{alias}-{bypass}-{B}-{N}".encode()))
    fp, push_c, sizes, offs, sym, idx = _push_case(rng, variant, alias, bypass, B, N)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, push_c, sizes, offs, fp, bypass, 4, alias=alias)
    assert perr == 0
    kw = dict(freq_precision=fp, bypass_coding=bypass, bypass_precision=4)
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, f"{variant}_alias_push" if alias else f"{variant}_push")(st, t(sym), t(idx), t(push_c), t(sizes),
                                                                          t(offs), **kw)
    assert C.device_status() == 0
    assert same_rows(st.cpu().numpy(), ref)


def wide_step_case(rng, B, N):
    """A table whose steps break the usual cdf shape: a start of -2^30 and a step of 2^24 - 1, far
    above 2^fp.  The reference still codes them (a 64-bit renormalisation bound, an exact division),
    and the states then leave [0, 2^31): rows of wrapped starts followed by the wide step drive
    the 32-bit states above 2^31 hundreds of times in a 400-symbol row."""
    base = -(1 << 30)
    wide = np.array([base, base + 50, base + 50 + (1 << 24) - 1, base + 50 + (1 << 24) + 99,
                     base + 50 + (1 << 24) + 199], np.int64).astype(np.int32)
    normal = np.array([0, 1000, 2000, 3000, 4096], np.int32)
    cdfs = np.stack([wide, normal])
    sizes = np.full(2, 5, np.int32)
    offs = np.zeros(2, np.int32)
    idx = (rng.random((B, N)) < 0.1).astype(np.int32)
    sym = rng.choice([0, 1, 2, 3], size=(B, N), p=[0.4, 0.4, 0.1, 0.1]).astype(np.int32)
    return 12, cdfs, sizes, offs, sym, idx


@pytest.mark.parametrize("kernel", PUSH_KERNELS)
@pytest.mark.parametrize("variant", VARIANTS)
def test_push_steps_wider_than_the_precision(C, kernel, variant, monkeypatch):
    """Steps wider than 2^fp go through the exact step code of every push kernel (the fast steps'
    reciprocal quotient holds only below 2^N); rows must equal the oracle's."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", kernel)
    B, N = 64, 400
    rng = np.random.default_rng(zlib.crc32(f"wide-{kernel}-{variant}".encode()))
    fp, cdfs, sizes, offs, sym, idx = wide_step_case(rng, B, N)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, offs, fp, False)
    assert perr == 0
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, f"{variant}_push")(st, t(sym), t(idx), t(cdfs), t(sizes), t(offs), freq_precision=fp,
                                  bypass_coding=False)
    assert C.device_status() == 0
    assert same_rows(st.cpu().numpy(), ref)


@pytest.mark.parametrize("kernel", PUSH_KERNELS)
@pytest.mark.parametrize("variant", VARIANTS)
def test_push_onto_popped_stream_keeps_old_words(C, kernel, variant, monkeypatch):
    """A stream pushed, popped back to its state and pushed again with fewer symbols needs no
    resize for the second push: the reference writes only the words it emits and leaves every
    other word of the row (the old words past the new length, and whatever the first resize left
    in the new columns) as it was.  From the same whole tensor, the second push must leave exactly
    the oracle's tensor (every push kernel, rows of 45 streams)."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", kernel)
    B, N1, N2 = 45, 400, 120
    rng = np.random.default_rng(zlib.crc32(f"repush-{kernel}-{variant}".encode()))
    fp, push_c, sizes, offs, sym1, idx1 = _push_case(rng, variant, False, False, B, N1)
    idx2 = rng.integers(0, push_c.shape[0], (B, N2)).astype(np.int32)
    sym2 = (rng.integers(0, sizes[idx2] - 1) + offs[idx2]).astype(np.int32)
    kw = dict(freq_precision=fp, bypass_coding=False, bypass_precision=4)
    ref, e = O.push(variant, O.init_stream(variant, B), sym1, idx1, push_c, sizes, offs, fp, False)
    assert e == 0
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, f"{variant}_push")(st, t(sym1), t(idx1), t(push_c), t(sizes), t(offs), **kw)
    assert same_rows(st.cpu().numpy(), ref)
    _, e = O.pop(variant, ref, idx1, push_c, sizes, offs, fp, False)
    assert e == 0
    getattr(C, f"{variant}_pop")(st, t(idx1), t(push_c), t(sizes), t(offs), **kw)
    assert same_rows(st.cpu().numpy(), ref)
    W = ref.shape[1]
    ref2, e = O.push(variant, st.cpu().numpy(), sym2, idx2, push_c, sizes, offs, fp, False)
    assert e == 0 and ref2.shape[1] == W  # no resize
    getattr(C, f"{variant}_push")(st, t(sym2), t(idx2), t(push_c), t(sizes), t(offs), **kw)
    assert C.device_status() == 0
    assert st.shape[1] == W and np.array_equal(st.cpu().numpy(), ref2)


@pytest.mark.parametrize("streams_per_block,chain_warps,prep_warps",
                         [("1", "1", "1"), ("64", "4", "4"), ("128", "4", "2"), ("37", "8", "8"), ("96", "2", "1")])
@pytest.mark.parametrize("variant", VARIANTS)
def test_ws_push_block_shapes(C, streams_per_block, chain_warps, prep_warps, variant, monkeypatch):
    """The warp-specialised push with forced block shapes (streams per block, chain and prep warp
    counts): one lane per stream on up to 8 chain warps, prep tasks shared unevenly among the prep
    threads.  Rows must match the oracle's exactly."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", "ws")
    monkeypatch.setenv("TORCH_ANS_B200_PUSHWS_STREAMS", streams_per_block)
    monkeypatch.setenv("TORCH_ANS_B200_PUSHWS_CHAIN_WARPS", chain_warps)
    monkeypatch.setenv("TORCH_ANS_B200_PUSHWS_PREP_WARPS", prep_warps)
    B, N = 300, 404
    rng = np.random.default_rng(zlib.crc32(f"wsshape-{streams_per_block}-{chain_warps}-{variant}".encode()))
    fp, push_c, sizes, offs, sym, idx = _push_case(rng, variant, False, True, B, N)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, push_c, sizes, offs, fp, True, 4)
    assert perr == 0
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, f"{variant}_push")(st, t(sym), t(idx), t(push_c), t(sizes), t(offs), freq_precision=fp,
                                  bypass_coding=True, bypass_precision=4)
    assert C.device_status() == 0
    assert same_rows(st.cpu().numpy(), ref)


@pytest.mark.parametrize("alias", [False, True])
@pytest.mark.parametrize("variant", VARIANTS)
def test_ws_push_many_blocks(C, variant, alias, monkeypatch):
    """The warp-specialised push at the launch shape of a large batch (8,192 streams: ~56 streams
    per block on every SM, more prep tasks than prep threads), with escapes: every row must match
    the oracle's.  Raw symbols and indexes pass through each block's shared-memory ring, so this
    checks the hand-over at the block shape the large workloads use."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", "ws")
    B, N = 8192, 96
    rng = np.random.default_rng(zlib.crc32(f"wsmany-{variant}-{alias}".encode()))
    fp, push_c, sizes, offs, sym, idx = _push_case(rng, variant, alias, True, B, N)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, push_c, sizes, offs, fp, True, 4, alias=alias)
    assert perr == 0
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    op = f"{variant}_alias_push" if alias else f"{variant}_push"
    getattr(C, op)(st, t(sym), t(idx), t(push_c), t(sizes), t(offs), freq_precision=fp, bypass_coding=True,
                   bypass_precision=4)
    assert C.device_status() == 0
    assert same_rows(st.cpu().numpy(), ref)


@pytest.mark.parametrize("ntables", [256, 257, 3000])
@pytest.mark.parametrize("variant", VARIANTS)
def test_ws_push_table_counts(C, variant, ntables, monkeypatch):
    """The warp-specialised push keeps 16 interleaved copies of the per-table {size, offset}
    records for up to 256 tables and one copy beyond: both sides of that limit, with escapes and
    table offsets, must give the oracle's rows."""
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", "ws")
    B, N = 300, 128
    rng = np.random.default_rng(zlib.crc32(f"wstables-{variant}-{ntables}".encode()))
    fp, cdfs, sizes, offs = _random_case(rng, variant, True, K=ntables, A=20)
    idx = rng.integers(0, ntables, (B, N)).astype(np.int32)
    sym = (rng.integers(-4, 26, (B, N)) + offs[idx]).astype(np.int32)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, offs, fp, True, 4)
    assert perr == 0
    st = getattr(C, f"{variant}_init_stream")(B).cuda()
    getattr(C, f"{variant}_push")(st, t(sym), t(idx), t(cdfs), t(sizes), t(offs), freq_precision=fp,
                                  bypass_coding=True, bypass_precision=4)
    assert C.device_status() == 0
    assert same_rows(st.cpu().numpy(), ref)


@pytest.mark.parametrize("kernel", PUSH_KERNELS)
@pytest.mark.parametrize("variant", VARIANTS)
def test_push_row_overflow_matches_oracle(kernel, variant, monkeypatch):
    """Rows too short for their words (a caller-sized buffer through the C ABI): every kernel keeps
    the words that fit, counts the rest, flags TANS_DEV_OVERFLOW and never writes past the row,
    exactly as the oracle's bounds-checked restatement does."""
    from torch_ans_b200 import capi
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", kernel)
    lib = capi.load()
    B, N = 40, 400
    rng = np.random.default_rng(zlib.crc32(f"ovf-{kernel}-{variant}".encode()))
    fp, push_c, sizes, offs, sym, idx = _push_case(rng, variant, False, False, B, N)
    init = O.init_stream(variant, B)
    W = init.shape[1] + 6  # room for a few words only
    host = np.zeros((B, W), np.int32)
    host[:, : init.shape[1]] = init
    ref = host.copy()
    err = O.lib().orc_push(O.VARIANTS[variant], 0, 1, O._ptr(ref), B, W, O._ptr(sym), O._ptr(idx), N,
                           O._ptr(push_c), push_c.shape[0], push_c.shape[1], O._ptr(sizes), O._ptr(offs), fp, 0, 4, 1)
    assert err & O.ERR_OVERFLOW
    # rows are contiguous, so a write past a row's end would land in the next row's length word;
    # guard words after the last row catch the rest
    guard = 8
    flat = torch.full((B * W + guard,), 0x5A5A5A5A, dtype=torch.int32, device="cuda")
    flat[: B * W] = t(host).reshape(-1)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    cs = torch.cuda.current_stream().cuda_stream
    s_d, i_d, c_d, z_d, o_d = t(sym), t(idx), t(push_c), t(sizes), t(offs)
    rc = lib.tans_push(capi.VARIANT[variant], 0, 1, flat.data_ptr(), B, W, s_d.data_ptr(), i_d.data_ptr(), N,
                       c_d.data_ptr(), c_d.shape[0], c_d.shape[1], z_d.data_ptr(), o_d.data_ptr(), fp, 0, 4, None, 0,
                       status.data_ptr(), cs)
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == err
    out = flat.cpu().numpy()
    assert np.all(out[B * W:] == 0x5A5A5A5A)
    assert np.array_equal(out[: B * W].reshape(B, W), ref)


def _heavy_tail_case(rng, K=6, A=300, fp=16):
    """Tables where most symbols have frequency 1 (long flat tails around a few large symbols), so
    many 16-cum buckets hold more than two symbols and the bucket layout falls back per step."""
    freqs = np.ones((K, A), np.int64)
    for k in range(K):
        big = rng.choice(A, 3, replace=False)
        share = rng.dirichlet(np.ones(3)) * ((1 << fp) - A)
        freqs[k, big] += np.floor(share).astype(np.int64)
        freqs[k, big[0]] += (1 << fp) - freqs[k].sum()
    cdfs = np.concatenate([np.zeros((K, 1), np.int64), np.cumsum(freqs, 1)], 1).astype(np.int32)
    sizes = np.full(K, A + 1, np.int32)
    offs = rng.integers(-8, 8, K).astype(np.int32)
    return fp, cdfs, sizes, offs


def _tail_combos():
    """The level-1 table fronts the bucket layout only."""
    return [pytest.param(kernel, layout, lookup, variant, id=f"{variant}-{lookup}-{layout}-{kernel}")
            for kernel in ("lean", "lean_l1", "fast")
            for layout in ("bucket_global", "split_global", "split_smem", "fused_smem")
            for lookup in ("search", "invcdf") for variant in VARIANTS
            if not (kernel == "lean_l1" and layout != "bucket_global")]


@pytest.mark.parametrize("kernel,layout,lookup,variant", _tail_combos())
def test_pop_heavy_tails_and_overrun(C, kernel, layout, lookup, variant, monkeypatch):
    """Unit-frequency tails (bucket entries that cannot describe their cum range, so those steps
    take the split tables or the exact step), symbols drawn uniformly over the alphabet (every
    tail symbol occurs), bad table indexes in the pop, and pops that run past the encoded words
    (underflow): outputs, final rows and error bits must all equal the oracle's.  "lean" and
    "lean_l1" run the lean kernels without and with the bucket layout's level-1 table in shared
    memory."""
    monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean" if kernel.startswith("lean") else kernel)
    monkeypatch.setenv("TORCH_ANS_B200_POP_L1", "1" if kernel == "lean_l1" else "0")
    monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", layout)
    rng = np.random.default_rng(zlib.crc32(f"tail-{kernel}-{layout}-{lookup}-{variant}".encode()))
    fp = 11 if layout.endswith("smem") else 16
    if variant == "rans32_16":
        fp = min(fp, 15)
    fp, cdfs, sizes, offs = _heavy_tail_case(rng, A=200 if fp < 16 else 300, fp=fp)
    pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
    K = cdfs.shape[0]
    B, N, extra = 50, 600, 8
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = (rng.integers(0, sizes[idx] - 1) + offs[idx]).astype(np.int32)
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, offs, fp, False)
    assert perr == 0
    # pop N + extra symbols with a few invalid indexes sprinkled in
    idx_pop = np.concatenate([idx, rng.integers(0, K, (B, extra)).astype(np.int32)], 1)
    bad = rng.random(idx_pop.shape) < 0.002
    idx_pop[bad] = K + 3
    ref_pop = ref.copy()
    dec_ref, derr = O.pop(variant, ref_pop, idx_pop, pop_c, sizes, offs, fp, False, lookup=lookup)
    assert derr & O.ERR_UNDERFLOW
    st = t(ref)
    dec = getattr(C, op_names(variant, 1, False, lookup)[1])(st, t(idx_pop), t(pop_c), t(sizes), t(offs),
                                                           freq_precision=fp, bypass_coding=False)
    assert C.device_status() == derr
    assert np.array_equal(dec.cpu().numpy(), dec_ref)
    assert same_rows(st.cpu().numpy(), ref_pop)


def _set_l1(monkeypatch, l1):
    """"0" / "1": level-1 table off / on at its default granularity; "1:b": on, 2^b cum values per
    entry."""
    on, _, bits = l1.partition(":")
    monkeypatch.setenv("TORCH_ANS_B200_POP_L1", on)
    if bits:
        monkeypatch.setenv("TORCH_ANS_B200_POP_L1_BITS", bits)


@pytest.mark.parametrize("iring", ["1", "0"])
@pytest.mark.parametrize("l1", ["0", "1", "1:10", "1:12"])
@pytest.mark.parametrize("lookup", ["search", "invcdf"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_bucket_pop_zero_offsets_tails_and_bad_rows(C, lookup, variant, l1, iring, monkeypatch):
    """The bucket-layout pop with every table offset zero (the kernel then skips the per-step
    offset read), a table whose last symbol covers whole buckets up to 2^fp, unit-frequency tails
    (marker buckets), bad indexes and underflow: identical to the oracle.  Then rows whose length
    points past the row's end (a corrupted length the reference would read past the row for): the
    bucket pop must agree with the generic pop kernel, which takes the same exact step, and flag
    underflow.  With and without the level-1 table in shared memory, with the indexes through the
    shared-memory ring fed by bulk copies and on plain loads; level-1 entries of 2^8 (the default
    here), 2^10 and 2^12 cum values."""
    monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
    monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "bucket_global")
    _set_l1(monkeypatch, l1)
    monkeypatch.setenv("TORCH_ANS_B200_POP_IRING", iring)
    rng = np.random.default_rng(zlib.crc32(f"bucket0-{lookup}-{variant}".encode()))
    fp = FP[variant]
    fp, cdfs, sizes, _ = _heavy_tail_case(rng, K=5, A=300, fp=fp)
    # last table: the last symbol takes a large share, so its buckets run up to cum = 2^fp - 1
    f = np.diff(cdfs[-1].astype(np.int64))
    f[:] = 1
    f[-1] += (1 << fp) - f.sum() - 4000
    f[0] += 4000
    cdfs[-1] = np.concatenate([[0], np.cumsum(f)]).astype(np.int32)
    offs = np.zeros(cdfs.shape[0], np.int32)
    pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
    K = cdfs.shape[0]
    B, N, extra = 40, 800, 8
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = rng.integers(0, sizes[idx] - 1).astype(np.int32)
    last = idx == K - 1
    sym[last] = np.where(rng.random(last.sum()) < 0.7, sizes[K - 1] - 2, sym[last])
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, offs, fp, False)
    assert perr == 0
    idx_pop = np.concatenate([idx, rng.integers(0, K, (B, extra)).astype(np.int32)], 1)
    idx_pop[rng.random(idx_pop.shape) < 0.002] = -1
    ref_pop = ref.copy()
    dec_ref, derr = O.pop(variant, ref_pop, idx_pop, pop_c, sizes, offs, fp, False, lookup=lookup)
    assert derr & O.ERR_UNDERFLOW and derr & O.ERR_BAD_INDEX
    pop = op_names(variant, 1, False, lookup)[1]
    kw = dict(freq_precision=fp, bypass_coding=False)
    st = t(ref)
    dec = getattr(C, pop)(st, t(idx_pop), t(pop_c), t(sizes), t(offs), **kw)
    assert C.device_status(reset=True) == derr
    assert np.array_equal(dec.cpu().numpy(), dec_ref)
    assert same_rows(st.cpu().numpy(), ref_pop)
    # corrupted lengths: every fourth row claims more bytes than the row holds
    bad = ref.copy()
    bad[::4, 0] = (bad.shape[1] - 1) * 4 + 16
    outs = {}
    for kernel in ("lean", "generic"):
        monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", kernel)
        st = t(bad)
        d = getattr(C, pop)(st, t(idx), t(pop_c), t(sizes), t(offs), **kw)
        outs[kernel] = (d.cpu().numpy(), st.cpu().numpy(), C.device_status(reset=True))
    assert outs["lean"][2] == outs["generic"][2] and outs["lean"][2] & O.ERR_UNDERFLOW
    assert np.array_equal(outs["lean"][0], outs["generic"][0])
    assert np.array_equal(outs["lean"][1], outs["generic"][1])
    # the rows with intact lengths decode as before
    assert np.array_equal(outs["lean"][0][1::4], sym[1::4])


@pytest.mark.parametrize("nchunks", [1, 2, 16, 17, 33])
@pytest.mark.parametrize("iring", ["1", "0"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_bucket_pop_short_rows_and_ring_boundaries(C, variant, iring, nchunks, monkeypatch):
    """Rows of 1, 2, 16, 17 and 33 chunks of four symbols: the index ring's first fill, its
    half boundaries (16 chunks per half) and its refills at the row's end, against the oracle."""
    monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
    monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "bucket_global")
    monkeypatch.setenv("TORCH_ANS_B200_POP_L1", "0")
    monkeypatch.setenv("TORCH_ANS_B200_POP_IRING", iring)
    rng = np.random.default_rng(zlib.crc32(f"ring-{variant}-{nchunks}".encode()))
    fp = FP[variant]
    fp, cdfs, sizes, offs = _heavy_tail_case(rng, K=7, A=120, fp=fp)
    K = cdfs.shape[0]
    B, N = 37, 4 * nchunks
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = (rng.integers(0, sizes[idx] - 1) + offs[idx]).astype(np.int32)
    # uniform symbols over heavy tails cost ~fp bits each: on rows this short the worst-case
    # width rule leaves no slack, so the rows get preallocated room
    ref, perr = O.push(variant, O.init_stream(variant, B, preallocate_size=64), sym, idx, cdfs, sizes, offs, fp,
                       False)
    assert perr == 0
    st = t(ref)
    dec = getattr(C, f"{variant}_pop")(st, t(idx), t(cdfs), t(sizes), t(offs), freq_precision=fp,
                                       bypass_coding=False)
    assert C.device_status() == 0
    assert np.array_equal(dec.cpu().numpy(), sym)
    ref_pop = ref.copy()
    O.pop(variant, ref_pop, idx, cdfs, sizes, offs, fp, False)
    assert same_rows(st.cpu().numpy(), ref_pop)


@pytest.mark.parametrize("l1", ["0", "1", "1:11"])
@pytest.mark.parametrize("lookup", ["search", "invcdf"])
@pytest.mark.parametrize("variant", VARIANTS)
def test_bucket_pop_secondary_table_overflow(C, lookup, variant, l1, monkeypatch):
    """Tables whose symbols alternate between frequency 1 and 2 over most of the range: nearly half
    of the buckets hold several symbols that are not a unit run, more than the secondary per-cum
    table has room for, so some of them decode from secondary blocks and the rest through the
    exact step.  Both must give the oracle's bytes, with and without the level-1 table."""
    monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
    monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "bucket_global")
    _set_l1(monkeypatch, l1)
    rng = np.random.default_rng(zlib.crc32(f"secovf-{lookup}-{variant}".encode()))
    fp = FP[variant]
    A = 5000 if fp == 15 else 10000
    rows = []
    for k in range(2):
        f = np.where(np.arange(A) % 2 == 0, 1, 2).astype(np.int64)
        f[rng.integers(0, A)] += (1 << fp) - f.sum()
        rows.append(np.concatenate([[0], np.cumsum(f)]))
    cdfs = np.stack(rows).astype(np.int32)
    sizes = np.full(2, A + 1, np.int32)
    offs = np.array([0, 3], np.int32)
    pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
    B, N = 16, 400
    idx = rng.integers(0, 2, (B, N)).astype(np.int32)
    sym = (rng.integers(0, A, (B, N)) + offs[idx]).astype(np.int32)  # uniform: tail symbols everywhere
    ref, perr = O.push(variant, O.init_stream(variant, B), sym, idx, cdfs, sizes, offs, fp, False)
    assert perr == 0
    ref_pop = ref.copy()
    dec_ref, derr = O.pop(variant, ref_pop, idx, pop_c, sizes, offs, fp, False, lookup=lookup)
    assert derr == 0
    pop = op_names(variant, 1, False, lookup)[1]
    st = t(ref)
    dec = getattr(C, pop)(st, t(idx), t(pop_c), t(sizes), t(offs), freq_precision=fp, bypass_coding=False)
    assert C.device_status(reset=True) == 0
    assert np.array_equal(dec.cpu().numpy(), sym)
    assert same_rows(st.cpu().numpy(), ref_pop)


@pytest.mark.parametrize("case", ["valid", "not_power_of_two", "bad_sum", "oversize", "mixed"])
def test_alias_build_on_device_matches_host(C, case):
    """rans_alias_build_table on CUDA tables (the device builder, tans_alias_build_table) returns
    exactly the host builder's remap and table rows -- the rows the reference builds, including the
    partial or empty rows of tables whose cut condition fails."""
    rng = np.random.default_rng(zlib.crc32(f"alias-dev-{case}".encode()))
    fp, sp = 12, 5
    K, A = 6, 1 << sp
    pm = rng.random((K, A)) + 0.02
    cdfs = O.pmf_to_quantized_cdf((pm / pm.sum(1, keepdims=True)).astype(np.float32), fp)
    sizes = np.full(K, A + 1, np.int32)
    if case == "not_power_of_two":
        sizes[:] = A  # A - 1 symbols: the cut does not divide 2^fp into 2^sp cuts
    elif case == "bad_sum":
        cdfs[:, -1] -= 3
    elif case == "oversize":
        sizes[1] = cdfs.shape[1] + 5
        sizes[2] = -1
    elif case == "mixed":
        sizes[0] = A
        cdfs[3, -1] += 1
    host_remap, host_tab = C.rans_alias_build_table(torch.from_numpy(cdfs), torch.from_numpy(sizes), sp, fp)
    dev_remap, dev_tab = C.rans_alias_build_table(t(cdfs), t(sizes), sp, fp)
    assert dev_remap.is_cuda and dev_tab.is_cuda
    assert torch.equal(dev_remap.cpu(), host_remap) and torch.equal(dev_tab.cpu(), host_tab)
    if case == "valid":
        g_remap, g_tab, ok = O.alias_build_table(cdfs, sizes, sp, fp)
        assert ok == K and np.array_equal(host_remap.numpy(), g_remap) and np.array_equal(host_tab.numpy(), g_tab)


def test_alias_build_on_device_golden():
    """The golden alias tables made by the compiled reference, rebuilt on the device."""
    import glob
    import json
    import os
    from torch_ans_b200 import _C
    checked = 0
    for name in [n for n in G.coding_cases() if "alias" in n]:
        d = G.load(name)
        m = d["meta"]
        w = int(d["sizes"].max()) - 1  # the golden cases use one cut per symbol
        sp = int(np.log2(w))
        if (1 << sp) != w:
            continue
        remap, tab = _C.rans_alias_build_table(t(d["cdfs"]), t(d["sizes"]), sp, int(m["fp"]))
        assert np.array_equal(remap.cpu().numpy(), d["push_cdfs"]) and np.array_equal(tab.cpu().numpy(), d["pop_cdfs"])
        checked += 1
    here = os.path.join(os.path.dirname(__file__), "golden")
    for path in sorted(glob.glob(os.path.join(here, "*_alias_rejected.npz"))):
        z = np.load(path)
        meta = json.loads(str(z["meta"]))
        remap, tab = _C.rans_alias_build_table(t(z["cdfs"]), t(z["sizes"]), meta["sp"], meta["fp"])
        assert np.array_equal(remap.cpu().numpy(), z["remap"]) and np.array_equal(tab.cpu().numpy(), z["table"])
        checked += 1
    assert checked >= 6
