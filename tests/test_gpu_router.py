"""Router on the GPU (glmx_router) against the restatement (fto_router_select / fto_router_gate) and the published
routing fixture (tests/golden/router.npz, made by tests/golden/make_router_golden.py).

Selection: bit-exact (same experts in the same order, same weights) given the same fp32 logits. Gate linear: the
GPU sums in fp32 in an order of its own, so its logits are compared with the fp64-accumulated oracle within
4e-6 x max|logit|; the selection is then checked bit-exact on the GPU's own logits."""
import sys

import numpy as np
import pytest

from conftest import GOLDEN, load_golden

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def _cases():
    sys.path.insert(0, GOLDEN)
    import make_router_golden as M
    return M


@pytest.mark.parametrize("name", ["glm288", "grouped256", "nonorm160"])
def test_select_bit_exact_vs_oracle(oracle, dev, name):
    from glmx import Router, synth
    M = _cases()
    ntok, E, topk, ng, tg, norm, scale, wb, seed = M.CASES[name]
    logits, bias = synth.router_inputs(ntok, E, seed)
    b = bias if wb else None
    r = Router(None, None if b is None else torch.from_numpy(b).to(dev), topk, ng, tg, norm, scale, n_experts=E)
    sel, w = r.select(torch.from_numpy(logits).to(dev))
    want_sel, want_w = oracle.router_select(logits, b, topk, ng, tg, norm, scale)
    np.testing.assert_array_equal(sel.cpu().numpy(), want_sel)
    np.testing.assert_array_equal(w.cpu().numpy(), want_w)
    # the published routing picks the same experts
    d = load_golden("router")
    np.testing.assert_array_equal(np.sort(sel.cpu().numpy(), axis=1), d[name + "_sel"])
    # int64 ids and fp16 weights (the reference hook's dtypes) are the same values, converted
    sel64, w16 = r.select(torch.from_numpy(logits).to(dev), sel_dtype=torch.int64, w_dtype=torch.float16)
    np.testing.assert_array_equal(sel64.cpu().numpy(), want_sel.astype(np.int64))
    np.testing.assert_array_equal(w16.cpu().numpy(), want_w.astype(np.float16))


def test_select_ties_and_large_batch(oracle, dev):
    from glmx import Router, synth
    r = Router(None, None, 8, 1, 1, True, 1.0, n_experts=288)
    sel, w = r.select(torch.zeros((3, 288), device=dev))
    np.testing.assert_array_equal(sel.cpu().numpy(), np.tile(np.arange(8, dtype=np.int32), (3, 1)))
    np.testing.assert_array_equal(w.cpu().numpy(), np.full((3, 8), np.float32(0.125)))
    # a prefill-sized batch with coarse logits (many exact ties) and a bias
    logits, bias = synth.router_inputs(4096, 288, 7011)
    logits = np.round(logits * 4.0).astype(np.float32) / 4.0
    r = Router(None, torch.from_numpy(bias).to(dev), 8, 1, 1, True, 1.0, n_experts=288)
    sel, w = r.select(torch.from_numpy(logits).to(dev))
    want_sel, want_w = oracle.router_select(logits, bias, 8, 1, 1, True, 1.0)
    np.testing.assert_array_equal(sel.cpu().numpy(), want_sel)
    np.testing.assert_array_equal(w.cpu().numpy(), want_w)


@pytest.mark.parametrize("ntok,H,E,zdt,wdt", [
    (16, 512, 288, torch.bfloat16, torch.bfloat16),      # the golden gate case
    (64, 6144, 288, torch.float16, torch.bfloat16),      # BASELINE geometry, decode batch
    (37, 6144, 288, torch.float32, torch.float32),       # ragged token block, fp32 everything
    (5, 256, 160, torch.bfloat16, torch.float16),
])
def test_gate_then_select(oracle, dev, ntok, H, E, zdt, wdt):
    from glmx import Router
    M = _cases()
    if (ntok, H, E) == (16, 512, 288):
        z, W = M.gate_inputs(**M.GATE)
    else:
        rng = np.random.default_rng(ntok * 1000 + H)
        z = rng.standard_normal((ntok, H)).astype(np.float32)
        W = (0.02 * rng.standard_normal((E, H))).astype(np.float32)
    zt = torch.from_numpy(z).to(dev).to(zdt)
    Wt = torch.from_numpy(W).to(dev).to(wdt)
    bias = torch.linspace(-0.1, 0.1, E, device=dev)
    r = Router(Wt, bias, 8, 1, 1, True, 1.0)
    for _ in range(2):                                    # the arrival counters reset themselves between calls
        sel, w, logits = r(zt)
        lg = logits.cpu().numpy()
        want_lg = oracle.router_gate(zt.float().cpu().numpy(), Wt.float().cpu().numpy())
        assert np.abs(lg - want_lg).max() <= 4e-6 * max(1.0, float(np.abs(want_lg).max()))
        want_sel, want_w = oracle.router_select(lg, bias.cpu().numpy(), 8, 1, 1, True, 1.0)
        np.testing.assert_array_equal(sel.cpu().numpy(), want_sel)
        np.testing.assert_array_equal(w.cpu().numpy(), want_w)
    if (ntok, H, E) == (16, 512, 288):
        d = load_golden("router")
        r0 = Router(Wt, None, 8, 1, 1, True, 1.0)
        sel, w, _ = r0(zt)
        np.testing.assert_array_equal(np.sort(sel.cpu().numpy(), axis=1), d["gate_sel"])


def test_router_feeds_the_layer(oracle, dev):
    """Router output straight into MoELayer.forward on the device equals the layer run on the oracle's picks."""
    from glmx import MoELayer, Router, _lib, synth
    H, I, E, ntok = 512, 256, 16, 12
    bank = synth.make_bank(H, I, E, shared=True, seed=1201)
    layer = MoELayer.from_bank(bank, device=dev)
    x = synth.make_x(ntok, H, 1202)
    xt = torch.from_numpy(x).to(dev)
    rng = np.random.default_rng(1203)
    W = torch.from_numpy((0.05 * rng.standard_normal((E, H))).astype(np.float32)).to(dev)
    r = Router(W, None, 4, 1, 1, True, 1.0)
    sel, w, logits = r(xt)
    got = layer.forward(xt, sel, w, mode=_lib.MODE_I16).cpu().numpy()
    osel, ow = oracle.router_select(logits.cpu().numpy(), None, 4, 1, 1, True, 1.0)
    want = layer.forward(xt, torch.from_numpy(osel).to(dev), torch.from_numpy(ow).to(dev), mode=_lib.MODE_I16).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    assert layer.check_device(ntok, 4) == 0
