"""The host-batch pipeline (torch_ans_b200.host_pipeline.HostStreamCoder) against the whole-batch
op path: the encoded bitstream must be byte-identical to push + stream_to_merged_tensor of the
same batch, and the decode must return the pushed symbols, for every variant, lookup, escape
mode and chunking (chunks that do not divide the length, chunks longer than the rows, chunks that
are not multiples of 4 and so take the generic kernels)."""
import zlib

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

VARIANTS = ["rans64", "rans32", "rans32_16"]


def _case(rng, variant, lookup, bypass, B, N):
    fp = 15 if variant == "rans32_16" else 16
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
        K, A = 5, 40
        pm = rng.integers(1, 1024, (K, A)).astype(np.float32)
        pm = np.concatenate([pm, np.ones((K, 1), np.float32)], 1)
        cdfs = O.pmf_to_quantized_cdf(pm / pm.sum(1, keepdims=True), fp)
        sizes = np.full(K, A + 2, np.int32)
        offs = rng.integers(-8, 8, K).astype(np.int32)
        push_c = cdfs
        pop_c = np.concatenate([cdfs, O.inverse_quantized_cdf(cdfs, fp)], 1) if lookup == "invcdf" else cdfs
        lo, hi = (-20, A + 20) if bypass else (0, A + 1)
    idx = rng.integers(0, K, (B, N)).astype(np.int32)
    sym = rng.integers(lo, hi, (B, N)).astype(np.int32)
    if not bypass:
        sym = (np.clip(sym, 0, sizes[idx] - 2) + offs[idx]).astype(np.int32)
    return fp, push_c, pop_c, sizes, offs, sym, idx


def _pinned(a):
    t = torch.empty(a.shape, dtype=torch.int32, pin_memory=True)
    t.copy_(torch.from_numpy(np.ascontiguousarray(a)))
    return t


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("lookup", ["search", "invcdf", "alias"])
@pytest.mark.parametrize("bypass", [False, True])
@pytest.mark.parametrize("chunk", [64, 100, 1000, 4096])
def test_pipeline_matches_whole_batch(variant, lookup, bypass, chunk):
    from torch_ans_b200 import _C
    from torch_ans_b200.host_pipeline import HostStreamCoder
    rng = np.random.default_rng(zlib.crc32(f"pipe-{variant}-{lookup}-{bypass}-{chunk}".encode()))
    B, N = 33, 1000
    fp, push_c, pop_c, sizes, offs, sym, idx = _case(rng, variant, lookup, bypass, B, N)
    kw = dict(freq_precision=fp, bypass_coding=bypass, bypass_precision=4)
    # whole-batch reference bytes through the op surface
    st = getattr(_C, f"{variant}_init_stream")(B).cuda()
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    getattr(_C, f"{variant}_alias_push" if lookup == "alias" else f"{variant}_push")(
        st, dev(sym), dev(idx), dev(push_c), dev(sizes), dev(offs), **kw)
    want = _C.stream_to_merged_tensor(st, 4, None).cpu()
    coder = HostStreamCoder(variant, torch.from_numpy(push_c), torch.from_numpy(pop_c), torch.from_numpy(sizes),
                            torch.from_numpy(offs), freq_precision=fp, bypass_coding=bypass, bypass_precision=4,
                            alias=lookup == "alias", lookup=lookup, chunk_symbols=chunk)
    h_sym, h_idx = _pinned(sym), _pinned(idx)
    got = coder.encode(h_sym, h_idx).clone()
    assert torch.equal(got, want)
    out = coder.decode(got, h_idx)
    assert coder.device_status() == 0
    assert np.array_equal(out.numpy(), sym)
    # a second round trip through the same coder reuses its buffers
    got2 = coder.encode(h_sym, h_idx)
    assert torch.equal(got2, want)
    assert np.array_equal(coder.decode(got2, h_idx).numpy(), sym)
