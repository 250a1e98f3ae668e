"""Failure detection on the GPU without a GPU fault.

Every hand-over wait in the warp-specialised push is bounded: when it runs out, the kernel sets
TANS_DEV_STALLED in the status word, tells the block's other warps through a shared abort flag,
lets its own copies land and returns -- no kernel is left waiting and the context stays usable.
The diagnostic variable TORCH_ANS_B200_WAIT_LIMIT sets the tries per wait; with 0 the first wait of
each warp gives up at once, which drives that path deterministically.  The test reads the status
bit on the host, then runs the same push with the normal limit on the same context and requires
the oracle's bytes.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

STALLED = 64


def _case():
    from torch_ans_b200 import workloads as W
    return W.laplace64(device="cuda", scale=1 / 4, length_scale=1 / 64)  # 16 streams x 1,024 symbols


def test_wait_that_runs_out_reports_stalled_and_context_survives(monkeypatch):
    from torch_ans_b200 import _C
    _C.set_sync_check(False)
    _C.device_status(reset=True)
    w = _case()
    B = w.symbols.shape[0]
    kw = dict(freq_precision=w.fp, bypass_coding=False)
    monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", "ws")
    monkeypatch.setenv("TORCH_ANS_B200_WAIT_LIMIT", "0")
    st = _C.rans64_init_stream(B, device="cuda")
    n0 = _C.launch_count()
    _C.rans64_push(st, w.symbols, w.indexes, w.cdfs, w.cdfs_sizes, w.offsets, **kw)
    assert _C.launch_count() > n0
    torch.cuda.synchronize()  # returns: no warp of the kernel is still waiting
    bits = _C.device_status(reset=True)
    assert bits & STALLED, f"status {bits}: the bounded wait did not report"
    # the rows of a stalled call are not valid, but the context is: the same push with the
    # normal wait limit runs and matches the oracle byte for byte
    monkeypatch.delenv("TORCH_ANS_B200_WAIT_LIMIT")
    st = _C.rans64_init_stream(B, device="cuda")
    _C.rans64_push(st, w.symbols, w.indexes, w.cdfs, w.cdfs_sizes, w.offsets, **kw)
    torch.cuda.synchronize()
    assert _C.device_status(reset=True) == 0
    ref, err = O.push("rans64", O.init_stream("rans64", B), w.symbols.cpu().numpy(), w.indexes.cpu().numpy(),
                      w.cdfs.cpu().numpy(), w.cdfs_sizes.cpu().numpy(), w.offsets.cpu().numpy(), w.fp, False)
    got = st.cpu().numpy()
    assert err == 0 and got.shape == ref.shape and np.array_equal(got[:, 0], ref[:, 0])
    assert b"".join(_C.rans_stream_to_byte_strings(st)) == b"".join(O.stream_to_byte_strings(ref))
    dec = _C.rans64_pop(st, w.indexes, w.cdfs, w.cdfs_sizes, w.offsets, **kw)
    assert torch.equal(dec, w.symbols) and _C.device_status() == 0
