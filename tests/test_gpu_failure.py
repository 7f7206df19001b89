"""Failure detection without a fault: the library's bounded device wait, run on a barrier that nothing completes,
gives up after its limit, reports the timeout bit and leaves the context usable (a forward right after is correct)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_bounded_wait_times_out_and_reports(oracle):
    from glmx import MoELayer, _lib, synth
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    _lib.check(lib.glmx_selftest_bounded_wait(3000, flag.data_ptr(), s.cuda_stream))
    e1.record(s)
    torch.cuda.synchronize(dev)
    assert int(flag.item()) == 1                         # the timeout bit glmx_check reports for a stalled forward
    assert e0.elapsed_time(e1) >= 3.0                    # it waited its limit, and no longer than the test
    # the context is intact: a forward right after is exact
    bank = synth.make_bank(256, 128, 3, shared=True, seed=961)
    layer = MoELayer.from_bank(bank, device=dev)
    x = synth.make_x(2, 256, 962)
    sel, w = synth.route_uniform(2, 3, 2, 963)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    got = layer.forward(t(x), t(sel), t(w), mode=_lib.MODE_I16).cpu().numpy()
    assert layer.check_device(2, 2) == 0
    np.testing.assert_array_equal(got, oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=2))


def test_peer_return_waits_are_bounded():
    """The owner's wait in the expert-parallel return gives up when a peer's flag never comes (here: world 2, only
    this rank's own flag set): error bit 16, out untouched, the context usable; with every flag set it sums in rank
    order."""
    import ctypes as C
    from glmx import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    world, rpr, H, seq = 2, 3, 256, 1
    recv = torch.randn((2, world, rpr, H), device=dev)
    flags = torch.zeros((2, world), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.full((rpr, H), 7.0, device=dev)
    flags[seq & 1, 0] = seq                              # rank 1's flag never arrives
    s = torch.cuda.current_stream(dev)
    _lib.check(lib.glmx_peer_reduce(recv.data_ptr(), flags.data_ptr(), world, rpr, H, seq, out.data_ptr(), _lib.F32,
                                    err.data_ptr(), s.cuda_stream))
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 16
    assert bool((out == 7.0).all())
    flags[seq & 1, 1] = seq
    err.zero_()
    _lib.check(lib.glmx_peer_reduce(recv.data_ptr(), flags.data_ptr(), world, rpr, H, seq, out.data_ptr(), _lib.F32,
                                    err.data_ptr(), s.cuda_stream))
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0
    want = recv[seq & 1, 0] + recv[seq & 1, 1]
    assert torch.equal(out, want)
