"""Pins the CPU restatement (oracle/ft_oracle.c) against fixtures produced by the reference's own ft_core.h
(tests/golden/make_golden.py) and by the reference's own hyper-connection kernels (tests/golden/make_hc_golden.py),
and the router restatement against the published GLM-4 MoE routing (tests/golden/make_router_golden.py). CPU only."""
import sys

import numpy as np
import pytest

from conftest import GOLDEN, golden_bank, load_golden, parity


def test_decode_known_answers(oracle):
    d = load_golden("decode_k3")
    got = oracle.decode_tiles(d["tiles"], 3)
    np.testing.assert_array_equal(got, d["decoded"])


def test_dense_matches_tilewise_decode(oracle):
    d = load_golden("decode_k3")
    tiles = d["tiles"]
    W = oracle.dense(tiles.reshape(-1), 3, 16, 16 * tiles.shape[0])
    dec = W.reshape(16, tiles.shape[0], 16).transpose(1, 0, 2).astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(dec, d["decoded"])


@pytest.mark.parametrize("name", ["moe_small", "moe_baseline"])
def test_fp64_expert_bit_exact(oracle, name):
    """The restatement's expert equals the reference's fp64 ref_expert (ft_core.h:1684-1691) bit for bit."""
    d = load_golden(name)
    b = golden_bank(d)
    for tag in d["cases"]:
        x = d[f"{tag}_x"]
        e0 = int(d[f"{tag}_sel"][0, 0])
        np.testing.assert_array_equal(oracle.expert(b, e0, x[0], mode=1)[0], d[f"{tag}_expert0_fp64"])
        np.testing.assert_array_equal(oracle.expert(b, b.E, x[0], mode=1)[0], d[f"{tag}_shared_fp64"])


@pytest.mark.parametrize("name", ["moe_small", "moe_baseline"])
def test_layer_vs_reference_fp32_kernel(oracle, name):
    """Whole layer against the reference's AVX2 moe_forward (fp32 accumulation, EXACT and AFFINE) and the band
    schedule. These reference kernels carry fp32 accumulation noise that the fp16 rounding points amplify: at
    H=6144 they sit 2.5-3e-3 x RMS (max-abs) away from the reference's own fp64 ref_expert, which the oracle
    reproduces bit for bit. The bound here is that measured noise floor, not the product's parity bar."""
    d = load_golden(name)
    b = golden_bank(d)
    for tag in d["cases"]:
        x, sel, w = d[f"{tag}_x"], d[f"{tag}_sel"], d[f"{tag}_w"]
        exact = oracle.moe_forward(b, x, sel, w, mode=1)
        affine = oracle.moe_forward(b, x, sel, w, mode=0)
        for key, ref in ((f"{tag}_exact", exact), (f"{tag}_band_exact", exact), (f"{tag}_affine", affine)):
            mx, rr = parity(d[key], ref)
            assert rr < 1e-3 and mx < 6e-3, (key, mx, rr)


def test_grouping_matches_reference_jobs(oracle):
    """Canonical expert-major rows hold exactly the reference's jobs (ft_core.h:1344-1349): same expert, same tokens in
    the same order, same weights, in chunks of MAXM = 8."""
    rng = np.random.default_rng(5)
    for ntok, topk, E in ((1, 8, 288), (7, 8, 16), (64, 8, 288), (40, 4, 5)):
        sel = np.stack([rng.permutation(E)[:topk] for _ in range(ntok)]).astype(np.int32)
        sel[rng.random(sel.shape) < 0.05] = -1
        w = rng.random(sel.shape).astype(np.float32)
        g = oracle.group(sel, w, E)
        jobs = oracle.jobs_ref(sel, w, E)
        canon = []
        for e in range(E):
            r0, r1 = g["offsets"][e], g["offsets"][e + 1]
            for c in range(r0, r1, 8):
                rows = range(c, min(c + 8, r1))
                canon.append((e, [int(g["row_token"][r]) for r in rows], [float(g["row_weight"][r]) for r in rows]))
        assert sorted(canon) == sorted(jobs)
        for p in range(ntok * topk):
            r = g["pick_row"][p]
            if sel.reshape(-1)[p] < 0:
                assert r == -1
            else:
                assert g["row_pick"][r] == p and g["row_token"][r] == p // topk


def test_i16_restatement_bit_exact_vs_reference(oracle):
    """The I16 restatement equals the reference's own mode 2 (moe_forward, ft_core.h) bit for bit on single-pick
    routes (layer output = one expert's output) and up to the combine's summation order on multi-pick routes."""
    d = load_golden("moe_i16_h4096")
    b = golden_bank(d)
    x, sel = d["single_x"], d["single_sel"]
    for t in range(x.shape[0]):
        np.testing.assert_array_equal(oracle.expert_i16(b, int(sel[t, 0]), x[t])[0], d["single_i16"][t])
    got = oracle.moe_forward(b, d["multi_x"], d["multi_sel"], d["multi_w"], mode=2)
    mx, rr = parity(got, d["multi_i16"])
    assert mx < 1e-6 and rr < 1e-7, (mx, rr)


def test_hc_apply_restatement(oracle):
    """fto_hc_apply against the same update in float64 (it differs only by fp32 rounding of each fma step)."""
    rng = np.random.default_rng(3)
    R, D = 3, 64
    x = rng.standard_normal((R, 4, D)).astype(np.float32)
    y = rng.standard_normal((R, D)).astype(np.float32)
    post = rng.random((R, 4)).astype(np.float32)
    comb = rng.standard_normal((R, 4, 4)).astype(np.float32)
    got = oracle.hc_apply(x, y, post, comb)
    want = post.astype(np.float64)[:, :, None] * y.astype(np.float64)[:, None, :] + \
        np.einsum("rhg,rhd->rgd", comb.astype(np.float64), x.astype(np.float64))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(x, oracle.hc_apply(x, y, post, comb) * 0 + x)      # input untouched


@pytest.mark.parametrize("case", ["apply_h", "apply_f"])
def test_hc_apply_pinned_to_reference_kernel(oracle, case):
    """fto_hc_apply equals the stream-stack update of the reference's own k_apply_partials (glm53/k_hcfuse.py:62-91,
    run by tests/golden/make_hc_golden.py) bit for bit, y given as fp16 and as fp32."""
    d = load_golden("hc_ref")
    got = oracle.hc_apply(d[f"{case}_x"], d[f"{case}_y"], d[f"{case}_post"], d[f"{case}_comb"])
    np.testing.assert_array_equal(got, d[f"{case}_xout"])


@pytest.mark.parametrize("case", ["apply_h", "apply_f", "mix_only", "final_h", "final_b"])
def test_hc_mix_partials_pinned_to_reference_kernel(oracle, case):
    """fto_hc_mix_partials equals the reference's hc_mix_partials (k_apply_partials, glm53/k_hcfuse.py:92-126) bit for
    bit, on the stack after its update (or as given, mix only)."""
    d = load_golden("hc_ref")
    stack = d[f"{case}_xout"] if f"{case}_xout" in d else d[f"{case}_x"]
    if case.startswith("final"):
        sys.path.insert(0, GOLDEN)
        import make_hc_golden as M
        c = [f for f in M.FINAL_CASES if f[0] == case][0]
        fn = M.inputs_final(c[1], c[2], c[6])[1]
    else:
        fn = d[f"{case}_fn"]
    np.testing.assert_array_equal(oracle.hc_mix_partials(stack, fn), d[f"{case}_part"])


@pytest.mark.parametrize("case", ["final_h", "final_b"])
def test_hc_finalize_restatement_vs_reference_kernel(oracle, case):
    """fto_hc_finalize_norm (plain fp32 math) against the reference's finalize_norm (fast intrinsics: __expf,
    __fdividef, rsqrtf, a few ulp each, 20 Sinkhorn rounds): post and comb within 1e-5 relative, the normalised fp16
    row within two fp16 steps of the reference's value (one rounding flip, which may cross a binade)."""
    d = load_golden("hc_ref")
    rms_eps, hc_eps, iters, n_eps, cbias, cscale = d[f"{case}_args"].tolist()
    post, comb, out = oracle.hc_finalize_norm(d[f"{case}_x"], d[f"{case}_part"], d[f"{case}_base"], d[f"{case}_scale"],
                                              d[f"{case}_nw"], rms_eps, hc_eps, int(iters), n_eps, cbias, cscale)
    np.testing.assert_allclose(post, d[f"{case}_post"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(comb, d[f"{case}_comb"], rtol=1e-5, atol=1e-7)
    ref = d[f"{case}_out"].astype(np.float32)
    step = np.abs(np.spacing(ref.astype(np.float16))).astype(np.float32)
    assert np.all(np.abs(out.astype(np.float32) - ref) <= 2 * step)


def _router_case(name):
    sys.path.insert(0, GOLDEN)
    import make_router_golden as M
    return M


def test_router_restatement_vs_published_routing(oracle):
    """The router restatement (fto_router_select / fto_router_gate) against the GLM-4 MoE routing as transformers runs
    it (tests/golden/make_router_golden.py): the same experts for every token, weights within 8 fp32 ulps (the
    published code sums the 8 weights in an order of its own and uses fp32 sigmoid)."""
    from glmx import synth
    M = _router_case("router")
    d = load_golden("router")
    for name, (ntok, E, topk, ng, tg, norm, scale, wb, seed) in M.CASES.items():
        logits, bias = synth.router_inputs(ntok, E, seed)
        sel, w = oracle.router_select(logits, bias if wb else None, topk, ng, tg, norm, scale)
        order = np.argsort(sel, axis=1, kind="stable")
        np.testing.assert_array_equal(np.take_along_axis(sel, order, 1), d[name + "_sel"], err_msg=name)
        np.testing.assert_allclose(np.take_along_axis(w, order, 1), d[name + "_w"], rtol=1e-6, atol=0, err_msg=name)
        # picks in descending choice score (c = sigmoid + bias)
        c = 1.0 / (1.0 + np.exp(-logits.astype(np.float64))) + (bias if wb else 0.0)
        cs = np.take_along_axis(c, sel, 1)
        assert (np.diff(cs, axis=1) <= 0).all(), name
    z, W = M.gate_inputs(**M.GATE)
    logits = oracle.router_gate(z, W)
    np.testing.assert_allclose(logits, d["gate_logits"], rtol=0, atol=2e-5 * float(np.abs(d["gate_logits"]).max()))
    sel, w = oracle.router_select(logits, None, 8, 1, 1, True, 1.0)
    order = np.argsort(sel, axis=1, kind="stable")
    np.testing.assert_array_equal(np.take_along_axis(sel, order, 1), d["gate_sel"])
    np.testing.assert_allclose(np.take_along_axis(w, order, 1), d["gate_w"], rtol=1e-6, atol=0)


def test_router_restatement_ties_and_groups(oracle):
    """Equal scores go to the smaller expert id; experts outside the kept groups are never picked while a kept group
    still has candidates."""
    logits = np.zeros((2, 16), np.float32)
    sel, w = oracle.router_select(logits, None, 4, 1, 1, True, 1.0)
    np.testing.assert_array_equal(sel, [[0, 1, 2, 3]] * 2)
    np.testing.assert_array_equal(w, np.full((2, 4), np.float32(0.25)))
    logits = np.full((1, 16), -3.0, np.float32)
    logits[0, [1, 9]] = 4.0                      # group 0 (ids 0..7) and group 1 (8..15): both have one big score
    logits[0, 10] = 3.0                          # group 1 has the larger top-2 sum
    sel, _ = oracle.router_select(logits, None, 3, 2, 1, False, 1.0)
    assert set(sel[0].tolist()) <= set(range(8, 16)) and sel[0, 0] == 9 and sel[0, 1] == 10


def test_router_sigmoid_error_bound(oracle):
    """The router's fp32 sigmoid (own Cody-Waite exp, identical fp32 steps on the CPU and the GPU) stays within 2.5 ulp
    of the exact value wherever the result is a normal fp32 number (x >= -87; below that, like torch's fp32 sigmoid,
    it returns 0 once e^-x overflows), and is exact at the ends."""
    x = np.concatenate([np.linspace(-87, 95, 400001, dtype=np.float32),
                        np.random.default_rng(5).standard_normal(200000).astype(np.float32) * 4])
    s = oracle.router_sigmoid(x).astype(np.float64)
    t = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    ulp = np.spacing(t.astype(np.float32)).astype(np.float64)
    assert (np.abs(s - t) / ulp).max() <= 2.5
    ends = oracle.router_sigmoid(np.array([0.0, 100.0, -100.0, np.inf, -np.inf], np.float32))
    np.testing.assert_array_equal(ends, np.array([0.5, 1.0, 0.0, 1.0, 0.0], np.float32))
    assert np.isnan(oracle.router_sigmoid(np.array([np.nan], np.float32))[0])
