"""Hyper-connection epilogue (glmx_moe_forward_hc): the stream-stack update that follows the MoE sublayer, fused into
the combine, against the oracle's restatement of the reference's hc_apply on the layer output the GPU produces
(bit for bit), on every path: I16, EXACT GEMV, EXACT tensor-core GEMM."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("mode_name,ntok,y_half", [("i16", 5, True), ("exact_gemv", 5, False), ("exact_gemm", 160, True)])
def test_forward_hc_bit_exact(oracle, mode_name, ntok, y_half):
    from glmx import MoELayer, _lib, synth
    dev = torch.device("cuda", 0)
    mode = {"i16": _lib.MODE_I16, "exact_gemv": _lib.MODE_EXACT | _lib.PATH_GEMV,
            "exact_gemm": _lib.MODE_EXACT | _lib.PATH_GEMM}[mode_name]
    H, I, E, topk = 512, 256, 6, 4
    bank = synth.make_bank(H, I, E, shared=True, seed=951)
    layer = MoELayer.from_bank(bank, device=dev)
    rng = np.random.default_rng(952)
    x = synth.make_x(ntok, H, 953)
    sel, w = synth.route_uniform(ntok, E, topk, 954)
    xs = rng.standard_normal((ntok, 4, H)).astype(np.float32)
    post = rng.random((ntok, 4)).astype(np.float32) * 2
    comb = rng.standard_normal((ntok, 4, 4)).astype(np.float32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    y = layer.forward(t(x), t(sel), t(w), mode=mode).cpu().numpy()
    yy = y.astype(np.float16).astype(np.float32) if y_half else y
    want = oracle.hc_apply(xs, yy, post, comb)
    hx = t(xs)
    layer.forward_hc(t(x), t(sel), t(w), hx, t(post), t(comb), y_half=y_half, mode=mode)
    assert layer.check_device(ntok, topk) == 0
    np.testing.assert_array_equal(hx.cpu().numpy(), want)
