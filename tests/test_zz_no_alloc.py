"""Tests of tans_push_noalloc, the encode entry point for callers that cannot allocate device
memory (a host whose device memory belongs to another allocator, a plugin limited to the buffers
it is handed, a serving loop that must not allocate).  Instead of a workspace from the caller or
from cudaMalloc it uses a fixed scratch array inside the library, shared by every call.

The GPU test calls it through the C ABI and requires its output to equal tans_push's byte for
byte on two calls in a row, the second one running on the scratch contents the first one left.
This file is collected last so a stop-at-first-failure run has already run everything else."""
import ctypes

import numpy as np
import pytest
import torch

from tests import golden_cases as G

TOO_LARGE = 4


INVALID = 1
LIMIT = 8 << 20
# Host-only calls below pass a placeholder address for each buffer: the argument and size checks
# run on the host and return before anything is read or launched.
FAKE = ctypes.c_void_p(4096)


def test_noalloc_rejects_tables_beyond_its_scratch():
    """The size check happens on the host before any device work (no GPU needed)."""
    from torch_ans_b200 import capi
    lib = capi.load()
    # 4,096 tables x 4,096 entries x 16 bytes = 256 MiB of encode tables > the 8 MiB scratch
    rc = lib.tans_push_noalloc(0, 0, 1, FAKE, 1, 3, FAKE, FAKE, 4, FAKE, 4096, 4097, FAKE, None, 16, 0, 4, None, None)
    assert rc == TOO_LARGE
    assert lib.tans_status_string(rc) == b"problem larger than the entry point supports"
    # one table whose row is one entry wider than the limit allows (fp 19: 2^19 + 1 entries)
    rc = lib.tans_push_noalloc(0, 0, 1, FAKE, 1, 3, FAKE, FAKE, 4, FAKE, 1, (1 << 19) + 2, FAKE, None, 19, 0, 4, None,
                               None)
    assert rc == TOO_LARGE


def test_noalloc_reports_invalid_arguments_before_size():
    """Invalid arguments get tans_push's error code, whatever the table size."""
    from torch_ans_b200 import capi
    lib = capi.load()
    big = (4096, 4097)
    assert lib.tans_push_noalloc(0, 0, 3, FAKE, 1, 3, FAKE, FAKE, 4, FAKE, *big, FAKE, None, 16, 0, 4, None,
                                 None) == INVALID  # 3 interleaved states
    assert lib.tans_push_noalloc(0, 0, 1, None, 1, 3, FAKE, FAKE, 4, FAKE, *big, FAKE, None, 16, 0, 4, None,
                                 None) == INVALID  # no stream
    assert lib.tans_push_noalloc(1, 0, 1, FAKE, 1, 3, FAKE, FAKE, 4, FAKE, *big, FAKE, None, 24, 0, 4, None,
                                 None) == INVALID  # fp above rans32's 23


def _run(lib, name, w, push_cdfs, use_alias, stream0, status, ws=None, interleave=1):
    st = stream0.clone()
    B, N = w["sym"].shape
    K, Wc = push_cdfs.shape
    args = [w["variant"], int(use_alias), interleave, st.data_ptr(), B, st.shape[1], w["sym"].data_ptr(), w["idx"].data_ptr(), N,
            push_cdfs.data_ptr(), K, Wc, w["sizes"].data_ptr(), w["offs"].data_ptr(), w["fp"], int(w["bypass"]), 4]
    if name == "tans_push":
        args += [ws.data_ptr(), ws.numel()]
    args += [status.data_ptr(), torch.cuda.current_stream().cuda_stream]
    rc = getattr(lib, name)(*args)
    assert rc == 0, lib.tans_status_string(rc)
    return st


def _cases():
    from torch_ans_b200 import workloads as W
    out = []
    lap = W.laplace64(device="cuda", scale=1 / 4, length_scale=1 / 64)
    out.append(("laplace", lap.variant, lap.symbols, lap.indexes, lap.cdfs, lap.cdfs_sizes, lap.offsets, lap.fp, False,
                False))
    mix = W.mixture_invcdf(device="cuda", scale=1 / 64, length_scale=1 / 256)
    out.append(("mixture", mix.variant, mix.symbols, mix.indexes, mix.cdfs, mix.cdfs_sizes, mix.offsets, mix.fp, False,
                False))
    zipf = W.zipf_alias(device="cuda", scale=1 / 64, length_scale=1 / 1024)
    out.append(("zipf_alias", zipf.variant, zipf.symbols, zipf.indexes, zipf.push_cdfs, zipf.cdfs_sizes, zipf.offsets,
                zipf.fp, False, True))
    d = G.load("rans32_bypass")  # escape coding, odd length (generic kernel path)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    out.append(("bypass", "rans32", t(d["symbols"]), t(d["indexes"]), t(d["cdfs"]), t(d["sizes"]), t(d["offsets"]), 16,
                True, False))
    return out


@pytest.mark.gpu
def test_noalloc_push_matches_push_on_two_calls():
    from torch_ans_b200 import _C, capi
    lib = capi.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for label, variant, sym, idx, cdfs, sizes, offs, fp, bypass, alias in _cases():
        w = dict(variant=capi.VARIANT[variant], sym=sym.contiguous(), idx=idx.contiguous(), sizes=sizes, offs=offs, fp=fp,
                 bypass=bypass)
        B, N = sym.shape
        W_ = 1 + (8 if variant == "rans64" else 4) // 4 + (N * fp + 7) // 8 // 4 + (N if bypass else 0) + 2
        stream0 = getattr(_C, f"{variant}_init_stream")(B)
        stream0 = torch.cat([stream0, torch.zeros(B, W_ - stream0.shape[1], dtype=torch.int32)], 1).cuda()
        ws = torch.empty(lib.tans_push_workspace_size(w["variant"], cdfs.shape[0], cdfs.shape[1]) + 256,
                         dtype=torch.uint8, device="cuda")
        ref = _run(lib, "tans_push", w, cdfs, alias, stream0, status, ws)
        for call in range(2):
            got = _run(lib, "tans_push_noalloc", w, cdfs, alias, stream0, status)
            torch.cuda.synchronize()
            assert status.item() == 0, (label, call)
            g, r = got.cpu().numpy(), ref.cpu().numpy()
            assert np.array_equal(g[:, 0], r[:, 0]), (label, call)
            assert G.payload_bytes(g) == G.payload_bytes(r), (label, call)


def _stream0(variant, B, N, fp, bypass, interleave=1):
    from torch_ans_b200 import _C
    st = getattr(_C, f"{variant}_init_stream")(B, interleave)
    W_ = st.shape[1] + (N * fp + 7) // 8 // 4 + (N if bypass else 0) + 2
    return torch.cat([st, torch.zeros(B, W_ - st.shape[1], dtype=torch.int32)], 1).cuda()


def _compare(lib, label, w, cdfs, alias, stream0, status, interleave=1):
    ws = torch.empty(lib.tans_push_workspace_size(w["variant"], cdfs.shape[0], cdfs.shape[1]) + 256,
                     dtype=torch.uint8, device="cuda")
    ref = _run(lib, "tans_push", w, cdfs, alias, stream0, status, ws, interleave)
    for call in range(2):
        got = _run(lib, "tans_push_noalloc", w, cdfs, alias, stream0, status, interleave=interleave)
        torch.cuda.synchronize()
        assert status.item() == 0, (label, call)
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(g[:, 0], r[:, 0]), (label, call)
        assert G.payload_bytes(g) == G.payload_bytes(r), (label, call)


@pytest.mark.gpu
def test_noalloc_four_interleaved_states_match_push():
    from torch_ans_b200 import capi
    lib = capi.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for name in ("rans64_i4_plain", "rans32_i4_bypass"):
        d = G.load(name)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        m = d["meta"]
        w = dict(variant=capi.VARIANT[m["variant"]], sym=t(d["symbols"]), idx=t(d["indexes"]), sizes=t(d["sizes"]),
                 offs=t(d["offsets"]), fp=m["fp"], bypass=bool(m["bypass"]))
        B, N = d["symbols"].shape
        _compare(lib, name, w, t(d["cdfs"]), False, _stream0(m["variant"], B, N, m["fp"], bool(m["bypass"]), 4),
                 status, interleave=4)


def _wide_row_case(cdf_width):
    """One table of 256 symbols at fp 19 in a row `cdf_width` entries wide: the scratch a push needs
    grows with the row width (one entry per column up to 2^fp + 1), not with the table's size."""
    fp = 19
    g = torch.Generator().manual_seed(9)
    freq = torch.ones(256, dtype=torch.int64) + torch.multinomial(torch.ones(256), (1 << fp) - 256, replacement=True,
                                                                  generator=g).bincount(minlength=256)
    cdf = torch.zeros(cdf_width, dtype=torch.int32)
    cdf[1:257] = torch.cumsum(freq, 0).to(torch.int32)
    sym = torch.randint(0, 256, (4, 512), generator=g, dtype=torch.int32)
    return fp, cdf.reshape(1, -1).cuda(), sym.cuda()


@pytest.mark.gpu
def test_noalloc_at_the_scratch_limit_and_just_over():
    from torch_ans_b200 import capi
    lib = capi.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 256 bytes of table info + 524,272 entries x 16 bytes = exactly 8 MiB: runs and matches
    at_limit = (LIMIT - 256) // 16 + 1
    fp, cdf, sym = _wide_row_case(at_limit)
    assert lib.tans_push_workspace_size(0, 1, at_limit) == LIMIT
    w = dict(variant=0, sym=sym, idx=torch.zeros_like(sym), sizes=torch.tensor([257], dtype=torch.int32).cuda(),
             offs=torch.zeros(1, dtype=torch.int32).cuda(), fp=fp, bypass=False)
    _compare(lib, "at_limit", w, cdf, False, _stream0("rans64", 4, 512, fp, False), status)
    # one more entry: 16 bytes past the limit (rounded up to 256) -> rejected, nothing runs
    fp, cdf2, _ = _wide_row_case(at_limit + 1)
    st = _stream0("rans64", 4, 512, fp, False)
    before = st.clone()
    rc = lib.tans_push_noalloc(0, 0, 1, st.data_ptr(), 4, st.shape[1], sym.data_ptr(), w["idx"].data_ptr(), 512,
                               cdf2.data_ptr(), 1, cdf2.shape[1], w["sizes"].data_ptr(), w["offs"].data_ptr(), fp, 0, 4,
                               status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
    torch.cuda.synchronize()
    assert torch.equal(st, before)


@pytest.mark.gpu
def test_noalloc_empty_push_with_empty_rows():
    """No symbols and rows of width 0: succeeds like tans_push and leaves the stream as it was."""
    from torch_ans_b200 import capi
    lib = capi.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = _stream0("rans32", 3, 0, 16, False)
    before = st.clone()
    cs = torch.cuda.current_stream().cuda_stream
    for cdf_width in (0, 1):
        rc = lib.tans_push_noalloc(1, 0, 1, st.data_ptr(), 3, st.shape[1], None, None, 0, None, 0, cdf_width, None,
                                   None, 16, 0, 4, status.data_ptr(), cs)
        assert rc == 0
        rc = lib.tans_push(1, 0, 1, st.data_ptr(), 3, st.shape[1], None, None, 0, None, 0, cdf_width, None, None, 16,
                           0, 4, None, 0, status.data_ptr(), cs)
        assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(st, before) and status.item() == 0
