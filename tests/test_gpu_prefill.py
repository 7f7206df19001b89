"""Prefill path (tcgen05 tensor-core GEMM, EXACT mode) against the fp64 oracle and against the GEMV decode path.
Jobs of up to 128 rows per expert; ragged last jobs, the shared expert's rows, mixed bitrates, BASELINE geometry."""
import numpy as np
import pytest

from conftest import TOL_MAXABS_REL_RMS, assert_exact_mode, parity, reference_outputs

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


def _run(layer, x, sel, w, mode, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    out = layer.forward(t(x), t(sel), t(w), mode=mode).cpu().numpy()
    assert layer.check_device(x.shape[0], sel.shape[1]) == 0
    return out


@pytest.mark.parametrize("H,I,E,ntok,topk,bits", [
    (1024, 512, 6, 200, 4, (3, 3, 3)),       # 2 jobs per expert (128 + ragged), shared expert 200 rows
    (512, 256, 3, 90, 2, (2, 3, 4)),         # mixed bitrates, single ragged job per expert
    (1024, 256, 5, 130, 5, (4, 4, 2)),
])
def test_prefill_gemm_vs_oracle(oracle, dev, H, I, E, ntok, topk, bits):
    from glmx import MoELayer, _lib, synth
    bank = synth.make_bank(H, I, E, shared=True, bits=bits, seed=900 + H + E)
    layer = MoELayer.from_bank(bank, device=dev)
    x = synth.make_x(ntok, H, 901)
    sel, w = synth.route_uniform(ntok, E, topk, 902)
    sel[3, 0] = -1
    got = _run(layer, x, sel, w, _lib.MODE_EXACT | _lib.PATH_GEMM, dev)
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1)
    assert np.isfinite(got).all()
    assert_exact_mode(got, want, *reference_outputs(bank, x, sel, w), label=f"prefill {H}x{I} bits {bits}",
                      floor=tuple(bits) != (3, 3, 3))
    # the GEMV path on the same inputs: a different fp32 accumulation order, so only fp16 rounding flips differ
    gemv = _run(layer, x, sel, w, _lib.MODE_EXACT | _lib.PATH_GEMV, dev)
    mx, rr = parity(got, gemv)
    assert rr <= 1e-3 and mx <= 1e-2, (mx, rr)


def test_prefill_baseline_geometry(oracle, dev):
    """H=6144, I=1536, K=3 with skewed routing: one expert takes most rows (several full 128-row jobs)."""
    from glmx import MoELayer, _lib, synth
    E, ntok, topk = 4, 300, 2
    bank = synth.make_bank(6144, 1536, E, shared=True, seed=911)
    layer = MoELayer.from_bank(bank, device=dev)
    x = synth.make_x(ntok, 6144, 912)
    rng = np.random.default_rng(913)
    sel = np.stack([np.array([0, 1 + rng.integers(0, E - 1)]) for _ in range(ntok)]).astype(np.int32)
    w = rng.random((ntok, topk)).astype(np.float32)
    got = _run(layer, x, sel, w, _lib.MODE_EXACT | _lib.PATH_GEMM, dev)
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1)
    assert_exact_mode(got, want, *reference_outputs(bank, x, sel, w), label="prefill baseline geometry")


def test_prefill_auto_path_and_accumulate(oracle, dev):
    """From 12 rows per expert EXACT mode picks the GEMM path by itself; accumulate adds into fp16 out."""
    from glmx import MoELayer, _lib, synth
    H, I, E, ntok, topk = 512, 256, 2, 80, 2
    bank = synth.make_bank(H, I, E, shared=True, seed=921)
    layer = MoELayer.from_bank(bank, device=dev)
    x = synth.make_x(ntok, H, 922)
    sel, w = synth.route_uniform(ntok, E, topk, 923)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    auto = layer.forward(t(x), t(sel), t(w), mode=_lib.MODE_EXACT).cpu().numpy()
    forced = layer.forward(t(x), t(sel), t(w), mode=_lib.MODE_EXACT | _lib.PATH_GEMM).cpu().numpy()
    np.testing.assert_array_equal(auto, forced)
    base = torch.full((ntok, H), 0.5, dtype=torch.float16, device=dev)
    layer.forward(t(x), t(sel), t(w), mode=_lib.MODE_EXACT | _lib.PATH_GEMM, out=base, accumulate=True)
    want = (np.float16(0.5).astype(np.float32) + forced).astype(np.float16)
    np.testing.assert_array_equal(base.cpu().numpy(), want)


def test_i16_rejects_prefill_sizes(dev):
    from glmx import MoELayer, _lib, synth
    bank = synth.make_bank(256, 128, 2, shared=False, seed=931)
    layer = MoELayer.from_bank(bank, device=dev)
    ntok = 8193
    x = torch.zeros((ntok, 256), dtype=torch.float16, device=dev)
    sel = torch.zeros((ntok, 1), dtype=torch.int32, device=dev)
    w = torch.ones((ntok, 1), dtype=torch.float32, device=dev)
    with pytest.raises(_lib.GlmxError, match="decode mode"):
        layer.forward(x, sel, w, mode=_lib.MODE_I16)
    with pytest.raises(_lib.GlmxError, match="EXACT mode only"):
        layer.forward(x[:4], sel[:4], w[:4], mode=_lib.MODE_I16 | _lib.PATH_GEMM)
