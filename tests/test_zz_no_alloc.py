"""glmx_moe_forward_noalloc (scratch in the library's fixed device array) against glmx_moe_forward (caller workspace),
through the C ABI. Collected last so it also runs after every other GPU test has used the device."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup():
    from glmx import MoELayer, synth
    bank = synth.make_bank(6144, 1536, 12, shared=True, seed=41)
    layer = MoELayer.from_bank(bank, device="cuda")
    return layer


def _call_noalloc(layer, x, sel, w, mode, out):
    from glmx import _lib
    st = torch.cuda.current_stream().cuda_stream
    return layer.lib.glmx_moe_forward_noalloc(layer.h, x.data_ptr(), _lib.F16, x.shape[0], sel.data_ptr(), _lib.I32,
                                              w.data_ptr(), _lib.F32, sel.shape[1], mode, out.data_ptr(), _lib.F32, 0, st)


@pytest.mark.parametrize("mode", [1, 2])
def test_noalloc_matches_workspace_path(setup, mode):
    from glmx import _lib, synth
    layer = setup
    ntok, topk = 8, 8
    for call in range(2):                                        # two calls in a row, new inputs each time
        x = torch.from_numpy(synth.make_x(ntok, layer.H, 100 + 10 * mode + call)).cuda()
        s, w = synth.route_uniform(ntok, layer.E, topk, 200 + 10 * mode + call)
        sel, wt = torch.from_numpy(s).cuda(), torch.from_numpy(w).cuda()
        want = layer.forward(x, sel, wt, mode=mode)
        out = torch.full((ntok, layer.H), float("nan"), device="cuda")
        _lib.check(_call_noalloc(layer, x, sel, wt, mode, out))
        flags = C.c_int(-1)
        _lib.check(layer.lib.glmx_check_noalloc(layer.h, ntok, topk, torch.cuda.current_stream().cuda_stream, C.byref(flags)))
        assert flags.value == 0
        # the same kernels on the same inputs with only the scratch's address changed: the same bits
        np.testing.assert_array_equal(out.cpu().numpy(), want.cpu().numpy(), err_msg=f"mode {mode} call {call}")


def test_noalloc_scratch_holds_eight_tokens(setup):
    """The documented limit: 8 tokens x top-8 (+ the shared expert) at H=6144, I=1536 fit the built-in scratch."""
    from glmx import _lib
    assert setup.workspace_bytes(8, 8) <= _lib.NOALLOC_SCRATCH_BYTES


def test_noalloc_rejects_oversize(setup):
    from glmx import _lib
    layer = setup
    ntok, topk = 64, 8                                           # needs ~230 MB of scratch at this geometry
    assert layer.workspace_bytes(ntok, topk) > _lib.NOALLOC_SCRATCH_BYTES
    x = torch.zeros(ntok, layer.H, dtype=torch.float16, device="cuda")
    sel = torch.zeros(ntok, topk, dtype=torch.int32, device="cuda")
    w = torch.zeros(ntok, topk, dtype=torch.float32, device="cuda")
    out = torch.full((ntok, layer.H), 7.0, device="cuda")
    rc = _call_noalloc(layer, x, sel, w, 2, out)
    assert rc == _lib.E_WORKSPACE
    msg = layer.lib.glmx_last_error().decode()
    assert "built-in scratch holds" in msg and str(_lib.NOALLOC_SCRATCH_BYTES) in msg
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)                                 # nothing ran
