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


def test_noalloc_rejects_tables_beyond_its_scratch():
    """The size check happens on the host before any device work (no GPU needed)."""
    from torch_ans_b200 import capi
    lib = capi.load()
    # 4,096 tables x 4,096 entries x 16 bytes = 256 MiB of encode tables > the 8 MiB scratch
    rc = lib.tans_push_noalloc(0, 0, 1, None, 1, 3, None, None, 4, None, 4096, 4097, None, None, 16, 0, 4, None, None)
    assert rc == TOO_LARGE
    assert lib.tans_status_string(rc) == b"problem larger than the entry point supports"


def _run(lib, name, w, push_cdfs, use_alias, stream0, status, ws=None):
    st = stream0.clone()
    B, N = w["sym"].shape
    K, Wc = push_cdfs.shape
    args = [w["variant"], int(use_alias), 1, st.data_ptr(), B, st.shape[1], w["sym"].data_ptr(), w["idx"].data_ptr(), N,
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
