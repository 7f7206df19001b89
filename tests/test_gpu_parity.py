"""CUDA path vs the oracle through the C ABI: trellis decode and routing bit-exact, layer outputs within the
north-star bar (max-abs <= 2e-3 x RMS of the output)."""
import numpy as np
import pytest

from conftest import TOL_MAXABS_REL_RMS, assert_exact_mode, golden_bank, load_golden, parity, reference_outputs

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda", 0)


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_decode_tiles_bit_exact(oracle, dev, bits):
    from glmx import decode_tiles, synth
    n = 4096
    tiles = synth.splitmix_bytes(1000 + bits, n * 32 * bits).reshape(n, 32 * bits)
    tiles[:4] = np.stack([np.full(32 * bits, v, np.uint8) for v in (0x00, 0xFF, 0xAA, 0x55)])
    got = decode_tiles(torch.from_numpy(tiles).to(dev), bits).cpu().numpy().view(np.uint16)
    want = oracle.decode_tiles(tiles, bits)
    np.testing.assert_array_equal(got, want)


def test_decode_golden(dev):
    from glmx import decode_tiles
    d = load_golden("decode_k3")
    got = decode_tiles(torch.from_numpy(d["tiles"]).to(dev), 3).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, d["decoded"])


def _layer(bank, dev):
    from glmx import MoELayer
    return MoELayer.from_bank(bank, device=dev)


@pytest.mark.parametrize("ntok,topk,E", [(1, 8, 288), (8, 8, 288), (64, 8, 288), (5, 4, 6), (300, 8, 64), (0, 8, 16)])
def test_route_bit_exact(oracle, dev, ntok, topk, E):
    from glmx import synth
    bank = synth.make_bank(128, 128, E, shared=True, seed=1)
    layer = _layer(bank, dev)
    rng = np.random.default_rng(ntok * 7 + E)
    sel = np.zeros((ntok, topk), np.int32)
    for t in range(ntok):
        sel[t] = rng.permutation(E)[:topk]
    if ntok:
        sel[rng.random(sel.shape) < 0.03] = -1
        sel[rng.random(sel.shape) < 0.01] = E + 3        # out of range: skipped like sel < 0
    w = rng.random(sel.shape).astype(np.float32)
    for sel_t in (torch.from_numpy(sel), torch.from_numpy(sel.astype(np.int64))):
        r = layer.route(sel_t.to(dev), torch.from_numpy(w).to(dev))
        got = layer.route_arrays(r)
        sel_c = np.where((sel >= 0) & (sel < E), sel, -1)
        want = oracle.group(sel_c, w, E)
        P = want["P"]
        assert got["P"] == P and got["R"] == P + ntok
        np.testing.assert_array_equal(got["offsets"], want["offsets"])
        np.testing.assert_array_equal(got["row_token"][:P], want["row_token"])
        np.testing.assert_array_equal(got["row_weight"][:P], want["row_weight"])
        np.testing.assert_array_equal(got["row_pick"][:P], want["row_pick"])
        np.testing.assert_array_equal(got["pick_row"], want["pick_row"])
        # shared expert rows follow, one per token
        np.testing.assert_array_equal(got["row_token"][P:], np.arange(ntok))
        # jobs: <= 8 consecutive rows of one expert, covering every row once
        jobs = got["jobs"]
        cover = np.zeros(got["R"], np.int32)
        for e, r0, m, _ in jobs:
            assert 1 <= m <= 8
            cover[r0:r0 + m] += 1
            if e < E:
                assert want["offsets"][e] <= r0 and r0 + m <= want["offsets"][e + 1]
        assert (cover == 1).all()


@pytest.mark.parametrize("name", ["moe_small", "moe_baseline"])
def test_exact_layer_golden(oracle, dev, name):
    """EXACT mode on the golden reference layers (inputs of the reference's A/B harness) vs the fp64 oracle, judged
    against the reference's own fp32 EXACT kernels' outputs stored in the fixture (moe_forward and its band form)."""
    d = load_golden(name)
    bank = golden_bank(d)
    layer = _layer(bank, dev)
    for tag in d["cases"]:
        x, sel, w = d[f"{tag}_x"], d[f"{tag}_sel"], d[f"{tag}_w"]
        out = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev), mode=1)
        got = out.cpu().numpy()
        assert layer.check_device(*sel.shape) == 0
        want = oracle.moe_forward(bank, x, sel, w, mode=1)
        assert_exact_mode(got, want, d[f"{tag}_exact"], d[f"{tag}_band_exact"], label=f"{name}/{tag}")


@pytest.mark.parametrize("ntok", [1, 4])
def test_exact_layer_baseline_geometry(oracle, dev, ntok):
    """EXACT mode at BASELINE configs[1] shape (H=6144, I=1536, K=3, top-8 sigmoid router), 24 routed + shared,
    against the reference's fp32 EXACT kernels (moe_forward, moe_forward_band) run live on the same inputs."""
    from glmx import synth
    from oracle.oracle import with_shared_routes
    E = 24
    bank = synth.make_bank(6144, 1536, E, shared=True, seed=31)
    layer = _layer(bank, dev)
    x = synth.make_x(ntok, 6144, 41)
    sel, w = synth.route_uniform(ntok, E, 8, 51)
    out = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev), mode=1)
    got = out.cpu().numpy()
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1)
    ref_out, band_out = reference_outputs(bank, x, sel, w)
    assert_exact_mode(got, want, ref_out, band_out, label=f"baseline ntok={ntok}")


@pytest.mark.parametrize("bits", [(2, 2, 2), (4, 4, 4), (4, 4, 2), (2, 3, 4)])
def test_exact_layer_mixed_bitrate(oracle, dev, bits):
    """BASELINE configs[4] mixed K per projection in EXACT mode. K != 3 has no reference kernel: parity is against the
    parameterised restatement with the K=3 noise floor."""
    from glmx import synth
    E = 6
    bank = synth.make_bank(1024, 512, E, shared=True, bits=bits, seed=61)
    layer = _layer(bank, dev)
    x = synth.make_x(3, 1024, 71)
    sel, w = synth.route_uniform(3, E, 4, 81)
    got = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev),
                        mode=1).cpu().numpy()
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1)
    assert_exact_mode(got, want, label=str(bits), floor=True)


@pytest.mark.parametrize("ntok", [3, 40])
@pytest.mark.parametrize("H,I,bits", [(640, 384, (3, 3, 3)), (768, 384, (2, 3, 2)), (640, 512, (3, 3, 2)),
                                      (1024, 512, (3, 3, 4))])
def test_exact_stage_forms(oracle, dev, H, I, bits, ntok):
    """The EXACT GEMV streams two 128-input blocks per pipeline stage where its K (H for gate/up, I for down) is a
    multiple of 256 and its bitrates are at most 3, one block otherwise, and the split plan counts K splits in the
    same stages. These layers take the one-block form for one or both GEMVs (K an odd number of blocks, or K=4); at
    40 tokens the plan also splits K. Held to the fixed floors of the EXACT rule: the reference's non-band moe_forward
    does not serve H=640 (measured 3.8 x RMS from the restatement there), so it sets no bar."""
    from glmx import synth
    E = 6
    bank = synth.make_bank(H, I, E, shared=True, bits=bits, seed=H + I + ntok)
    layer = _layer(bank, dev)
    x = synth.make_x(ntok, H, 73 + ntok)
    sel, w = synth.route_uniform(ntok, E, 4, 83 + ntok)
    got = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev),
                        mode=1).cpu().numpy()
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1)
    assert_exact_mode(got, want, label=f"H={H} I={I} {bits} ntok={ntok}", floor=True)


def test_accumulate_and_fp16_out(oracle, dev):
    from glmx import synth
    E = 8
    bank = synth.make_bank(512, 256, E, shared=False, seed=91)
    layer = _layer(bank, dev)
    x = synth.make_x(4, 512, 92)
    sel, w = synth.route_uniform(4, E, 2, 93)
    xt, st, wt = (torch.from_numpy(a).to(dev) for a in (x, sel, w))
    base = torch.randn(4, 512, device=dev)
    for mode in (1, 2):
        acc = layer.forward(xt, st, wt, out=base.clone(), accumulate=True, mode=mode)
        plain = layer.forward(xt, st, wt, mode=mode)
        torch.testing.assert_close(acc, base + plain, rtol=0, atol=1e-6)
        h = layer.forward(xt, st, wt, out_dtype=torch.float16, mode=mode)
        torch.testing.assert_close(h.float(), plain.half().float(), rtol=0, atol=0)


# ---- I16 mode: bit-exact ---------------------------------------------------------------------------------------------

def test_i16_golden_reference_bit_exact(dev):
    """GPU I16 mode vs the reference's own moe_forward mode 2 at its geometry (H=4096, I=2048): bit-identical."""
    d = load_golden("moe_i16_h4096")
    bank = golden_bank(d)
    layer = _layer(bank, dev)
    x, sel, w = (torch.from_numpy(d[k]).to(dev) for k in ("single_x", "single_sel", "single_w"))
    got = layer.forward(x, sel, w, mode=2).cpu().numpy()
    assert layer.check_device(*sel.shape) == 0
    np.testing.assert_array_equal(got, d["single_i16"])
    x, sel, w = (torch.from_numpy(d[k]).to(dev) for k in ("multi_x", "multi_sel", "multi_w"))
    got = layer.forward(x, sel, w, mode=2).cpu().numpy()
    mx, rr = parity(got, d["multi_i16"])
    assert mx < 1e-6 and rr < 1e-7, (mx, rr)


@pytest.mark.parametrize("ntok,E,topk", [(1, 24, 8), (5, 24, 8), (16, 40, 8)])
def test_i16_baseline_geometry_bit_exact(oracle, dev, ntok, E, topk):
    """BASELINE geometry (H=6144, I=1536, K=3) with a shared expert: GPU I16 == oracle I16 restatement, every bit."""
    from glmx import synth
    bank = synth.make_bank(6144, 1536, E, shared=True, seed=131 + ntok)
    layer = _layer(bank, dev)
    x = synth.make_x(ntok, 6144, 141 + ntok)
    sel, w = synth.route_uniform(ntok, E, topk, 151 + ntok)
    got = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev),
                        mode=2).cpu().numpy()
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=2)
    mx, rr = parity(got, want)
    assert mx <= TOL_MAXABS_REL_RMS, (mx, rr)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("bits", [(2, 2, 2), (4, 4, 4), (2, 3, 4)])
def test_i16_mixed_bitrate_bit_exact(oracle, dev, bits):
    from glmx import synth
    E = 6
    bank = synth.make_bank(1024, 512, E, shared=True, bits=bits, seed=161)
    layer = _layer(bank, dev)
    x = synth.make_x(6, 1024, 171)
    sel, w = synth.route_uniform(6, E, 4, 181)
    got = layer.forward(torch.from_numpy(x).to(dev), torch.from_numpy(sel).to(dev), torch.from_numpy(w).to(dev),
                        mode=2).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=2))
