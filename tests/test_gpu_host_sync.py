"""Host synchronisation of the coding ops.

The reference's push reads the largest row length back to the host before its worst-case resize
(torch_ans/rans.hpp:106, ``.item()``).  Here a stream made on the device by
``rans*_init_stream(..., device=...)`` carries a host-side record of its lengths, so its push
resizes without reading the device; pops never read it.  These tests run the ops under
``torch.cuda.set_sync_debug_mode("error")``, which raises on any blocking device-to-host copy or
synchronisation torch performs, and check the bytes against the golden vectors.
"""
import numpy as np
import pytest
import torch

from tests import golden_cases as G

pytestmark = pytest.mark.gpu


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def C():
    from torch_ans_b200 import _C
    _C.set_sync_check(False)
    return _C


@pytest.mark.parametrize("name", ["rans64_plain", "rans32_bypass", "rans32_16_plain", "rans64_alias"])
def test_push_and_pop_on_device_stream_do_not_synchronise(C, name):
    d = G.load(name)
    m = d["meta"]
    v = m["variant"]
    push = f"{v}_alias_push" if m["alias_push"] else f"{v}_push"
    pop = {"alias": f"{v}_alias_pop", "invcdf": f"{v}_invcdf_pop", "search": f"{v}_pop"}[m["lookup"]]
    kw = dict(freq_precision=m["fp"], bypass_coding=bool(m["bypass"]), bypass_precision=m["bp"])
    sym, idx, pc, qc = t(d["symbols"]), t(d["indexes"]), t(d["push_cdfs"]), t(d["pop_cdfs"])
    sz, off = t(d["sizes"]), t(d["offsets"])
    torch.cuda.synchronize()
    st = getattr(C, f"{v}_init_stream")(sym.shape[0], device="cuda")
    torch.cuda.set_sync_debug_mode("error")
    try:
        getattr(C, push)(st, sym, idx, pc, sz, off, **kw)
        dec = getattr(C, pop)(st.clone(), idx, qc, sz, off, **kw)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    got = st.cpu().numpy()
    assert got.shape == d["pushed"].shape
    assert np.array_equal(got[:, 0], d["pushed"][:, 0])
    assert G.payload_bytes(got) == d["pushed_bytes"].tobytes()
    assert np.array_equal(dec.cpu().numpy(), d["decoded"])
    assert C.device_status() == 0


def test_stream_moved_from_cpu_is_resized_from_device_lengths(C):
    """A stream the host knows nothing about (made on the CPU, then moved) is resized from its
    device lengths, as the reference does: that read is a synchronisation the debug mode sees."""
    d = G.load("rans64_plain")
    st = C.rans64_init_stream(d["symbols"].shape[0]).cuda()
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        with pytest.raises(RuntimeError):
            C.rans64_push(st, t(d["symbols"]), t(d["indexes"]), t(d["cdfs"]), t(d["sizes"]), t(d["offsets"]),
                          freq_precision=16, bypass_coding=False)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    C.rans64_push(st, t(d["symbols"]), t(d["indexes"]), t(d["cdfs"]), t(d["sizes"]), t(d["offsets"]),
                  freq_precision=16, bypass_coding=False)
    got = st.cpu().numpy()
    assert got.shape == d["pushed"].shape and G.payload_bytes(got) == d["pushed_bytes"].tobytes()


def test_known_length_record_is_dropped_by_in_place_changes(C):
    """An in-place change through torch (version counter) or a coding op drops the host-side
    record: the next push reads the device lengths and still gets the reference's width."""
    d = G.load("rans64_streaming")
    cdfs, sizes, offs = t(d["cdfs"]), t(d["sizes"]), t(d["offsets"])
    st = C.rans64_init_stream(3, device="cuda")
    C.rans64_push(st, t(d["s2"]), t(d["i2"]), cdfs, sizes, offs, freq_precision=16)
    # second push onto the same stream: its lengths are no longer known on the host
    C.rans64_push(st, t(d["s1"]), t(d["i1"]), cdfs, sizes, offs, freq_precision=16)
    got = st.cpu().numpy()
    assert got.shape == d["after2"].shape and G.payload_bytes(got) == G.payload_bytes(d["after2"])
    st2 = C.rans64_init_stream(3, device="cuda")
    st2[:, 0] += 0  # an in-place torch op bumps the version counter
    C.rans64_push(st2, t(d["s2"]), t(d["i2"]), cdfs, sizes, offs, freq_precision=16)
    got = st2.cpu().numpy()
    assert got.shape == d["after1"].shape and G.payload_bytes(got) == G.payload_bytes(d["after1"])


def test_high_level_encode_does_not_synchronise_before_the_bytes(C):
    """TorchANSInterface.encode (tensor API) makes its stream on the device: no device read."""
    from torch_ans_b200.utils import TorchANSInterface
    g = torch.Generator().manual_seed(5)
    pmf = torch.randint(1, 100, (4, 16), generator=g, dtype=torch.int32)
    coder = TorchANSInterface(impl="rans64", freq_precision=12, device="cuda")
    coder.init_params(pmf, torch.full((4,), 16, dtype=torch.int32), torch.zeros(4, dtype=torch.int32))
    sym = torch.randint(0, 16, (2, 32), generator=g, dtype=torch.int32).cuda()
    idx = torch.randint(0, 4, (2, 32), generator=g, dtype=torch.int32).cuda()
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        stream = coder.encode(sym, dist_indexes=idx)
    finally:
        torch.cuda.set_sync_debug_mode(0)
    assert torch.equal(coder.decode(stream, dist_indexes=idx), sym)
