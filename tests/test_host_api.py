"""Host-side drop-in layers on CPU: the tier_* API mirror (argument checks, flow into the layer) and the
routing_fn / cpu_split_combine hooks (masking conventions, bypass conditions, fp16/fp32 combine), with fake layers."""
import numpy as np
import pytest
import torch

from glmx import hooks, tier


class FakeLayer:
    """Stands in for MoELayer on CPU: forward returns a fixed function of its inputs and records the call."""

    def __init__(self, H, I, E, ptrs, suh, svh, bits=(3, 3, 3), has_shared=False, act_limit=0.0, keep=(), device=None):
        self.H, self.E, self.has_shared, self.act_limit = H, E, has_shared, act_limit
        self.ptrs = torch.as_tensor(ptrs) if ptrs is not None else None
        self.device = torch.device("cpu")
        self.calls = []

    def forward(self, x, sel, w, mode=2):
        self.calls.append((x.clone(), sel.clone(), w.clone(), mode))
        return (x.float() * 0.5 + w.float().sum(1, keepdim=True)).contiguous()

    def set_act_limit(self, limit):
        self.act_limit = float(limit)


@pytest.fixture
def fake_tier(monkeypatch):
    monkeypatch.setattr(tier, "MoELayer", FakeLayer)
    tier.tier_reset()
    yield tier
    tier.tier_reset()


def _scales(E, H, I):
    h = lambda n: torch.ones(E, n, dtype=torch.float16)
    return h(H), h(I), h(H), h(I), h(I), h(H)


def test_tier_checks(fake_tier):
    T = fake_tier
    with pytest.raises(RuntimeError, match="init first"):
        T.tier_add_layer(0, torch.zeros(4, 3, dtype=torch.int64), *_scales(4, 256, 128))
    with pytest.raises(RuntimeError, match="multiples of 128"):
        T.tier_init(1, [0], None, None, None, None, 1, 200, 128, 2, 0)
    T.tier_init(1, [0], None, None, None, None, 1, 256, 128, 2, 0)
    with pytest.raises(RuntimeError, match="already initialised"):
        T.tier_init(1, [0], None, None, None, None, 1, 256, 128, 2, 0)
    with pytest.raises(RuntimeError, match="scale shapes"):
        T.tier_add_layer(0, torch.zeros(4, 3, dtype=torch.int64), *_scales(4, 128, 128))
    with pytest.raises(RuntimeError, match="scales"):
        s = list(_scales(4, 256, 128)); s[0] = s[0].float()
        T.tier_add_layer(0, torch.zeros(4, 3, dtype=torch.int64), *s)
    with pytest.raises(RuntimeError, match="not registered"):
        T.tier_forward(1, torch.zeros(1, 256), torch.zeros(1, 8, dtype=torch.int32), torch.zeros(1, 8), -1)
    T.tier_add_layer(1, torch.arange(12, dtype=torch.int64).reshape(4, 3), *_scales(4, 256, 128))
    with pytest.raises(RuntimeError, match="AFFINE"):
        T.tier_forward(1, torch.zeros(1, 256), torch.zeros(1, 8, dtype=torch.int32), torch.zeros(1, 8), 0)
    T.tier_start(0)
    with pytest.raises(RuntimeError, match="worker running"):
        T.tier_forward(1, torch.zeros(1, 256), torch.zeros(1, 8, dtype=torch.int32), torch.zeros(1, 8), 1)
    T.tier_stop()


def test_tier_forward_flow(fake_tier):
    T = fake_tier
    T.tier_init(1, [0], None, None, None, None, 1, 256, 128, 1, 0)
    sh = (torch.tensor([100, 101, 102]), [torch.ones(n, dtype=torch.float16) for n in (256, 256, 128)],
          [torch.ones(n, dtype=torch.float16) for n in (128, 128, 256)])
    T.tier_add_layer(0, torch.arange(12, dtype=torch.int64).reshape(4, 3), *_scales(4, 256, 128), shared=sh)
    layer = T.T.layers[0]
    assert layer.has_shared and layer.E == 4 and layer.ptrs.tolist()[-1] == [100, 101, 102]
    x = torch.randn(3, 256)
    sel = torch.tensor([[0, 1, -1, 2], [3, 3, 1, 0], [-1, -1, -1, -1]], dtype=torch.int32)
    w = torch.rand(3, 4)
    for mode, want in ((-1, 2), (1, 1), (2, 2)):
        out = T.tier_forward(0, x, sel, w, mode)
        assert layer.calls[-1][3] == want
        torch.testing.assert_close(out, x * 0.5 + w.sum(1, keepdim=True))
    st = T.tier_stats()
    assert st[0] == 3 and st[2] == 9 and st[1] == 3 * 4
    T.tier_set_act_limit(7.0)
    assert layer.act_limit == 7.0


class FakeModule:
    def __init__(self, sel, w):
        self._sel, self._w = sel, w
        self.combined = None

    def routing_fn(self, bsz, cfg, z, params):
        return self._sel.clone(), self._w.clone()

    def cpu_split_combine(self, fhs, cpu_partial, cpu_pending, shape):
        self.combined = fhs.clone()
        return fhs


@pytest.mark.parametrize("bsz", [1, 4, 16])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_hooks_route_and_combine(bsz, dtype):
    H, topk = 256, 8
    g = torch.Generator().manual_seed(bsz)
    sel = torch.randint(0, 64, (bsz, topk), generator=g, dtype=torch.int64)
    w = torch.rand(bsz, topk, generator=g).half()
    mod = FakeModule(sel, w)
    layer = FakeLayer(H, 128, 64, None, None, None)
    hooks.attach(mod, layer, mode=2)
    z = torch.randn(bsz, H, generator=g).half()
    so, wo = mod.routing_fn(bsz, None, z, {})
    x, s_seen, w_seen, mode = layer.calls[-1]
    assert mode == 2 and torch.equal(s_seen, sel) and torch.equal(w_seen, w) and torch.equal(x, z)
    assert torch.all(wo == 0) and wo.dtype == w.dtype
    assert torch.equal(so, sel) if bsz > 8 else torch.all(so == -1)
    fhs = torch.randn(bsz, H, generator=g).to(dtype)
    part = z.float() * 0.5 + w.float().sum(1, keepdim=True)
    want = (fhs.float() + part).half() if dtype == torch.float16 else fhs + part
    out = mod.cpu_split_combine(fhs, None, None, None)
    assert torch.equal(out, want) and torch.equal(mod.combined, want)
    # the partial is consumed: a second combine adds nothing
    again = mod.cpu_split_combine(out.clone(), None, None, None)
    assert torch.equal(again, want)


def test_hooks_bypass():
    sel = torch.zeros(2, 8, dtype=torch.int64)
    w = torch.ones(2, 8).half()
    mod = FakeModule(sel, w)
    layer = FakeLayer(256, 128, 8, None, None, None)
    hooks.attach(mod, layer, max_bsz=1)
    z = torch.zeros(2, 256).half()
    for bsz, params in ((2, {}), (1, {"autosplit_measure": True}), (1, {"tp_warmup": True})):
        so, wo = mod.routing_fn(bsz, None, z[:bsz], params)
        assert torch.equal(wo, w) and not layer.calls
        fhs = torch.ones(bsz, 256)
        assert torch.equal(mod.cpu_split_combine(fhs, None, None, None), fhs)


# ---- on-disk EXL3 adapter: hooks.layer_from_exllamav3 over exllamav3's per-expert tensors ----------------------------

class _Inner:
    def __init__(self, trellis, suh, svh):
        self.trellis, self.suh, self.svh = trellis, suh, svh


class _Linear:
    def __init__(self, inner):
        self.inner = inner


class _Multi:
    def __init__(self, linears):
        self.linears = linears


def fake_exl3_module(bank, device="cpu", act_limit=0.0):
    """A stand-in for exllamav3's BlockSparseMLP with the attributes the reference's cpu_tier reads
    (multi_{gate,up,down}.linears[e].inner.{trellis, suh, svh}, hidden/intermediate sizes, act_limit; glm53/cpu_tier.py:
    535-537, glm53/expert_cache.py:603-616): one trellis tensor per expert and projection (its own allocation, as
    exllamav3 loads them), suh/svh fp16 vectors."""
    import numpy as np

    class M:
        pass
    m = M()
    m.hidden_size, m.intermediate_size, m.act_limit = bank.H, bank.I, act_limit
    for p, name in enumerate(("multi_gate", "multi_up", "multi_down")):
        lins = []
        for e in range(bank.E):
            tr = torch.from_numpy(np.ascontiguousarray(bank.proj(e, p)).view(np.int16).copy()).to(device)
            lins.append(_Linear(_Inner(tr, torch.from_numpy(bank.suh[p][e].copy()).to(device),
                                       torch.from_numpy(bank.svh[p][e].copy()).to(device))))
        setattr(m, name, _Multi(lins))
    return m


def test_layer_from_exllamav3_tables(monkeypatch):
    """The adapter's pointer table, scales and sizes (host logic; the layer class is recorded, not built)."""
    from glmx import hooks, synth
    bank = synth.make_bank(256, 128, 5, shared=False, seed=3)
    m = fake_exl3_module(bank, act_limit=10.0)
    seen = {}

    class Rec:
        def __init__(self, H, I, E, ptrs, suh, svh, **kw):
            seen.update(H=H, I=I, E=E, ptrs=ptrs, suh=suh, svh=svh, **kw)
    monkeypatch.setattr(hooks, "MoELayer", Rec)
    hooks.layer_from_exllamav3(m, device="cpu")
    assert (seen["H"], seen["I"], seen["E"]) == (256, 128, 5) and seen["act_limit"] == 10.0 and not seen["has_shared"]
    for e in range(5):
        for p, name in enumerate(("multi_gate", "multi_up", "multi_down")):
            inner = getattr(m, name).linears[e].inner
            assert int(seen["ptrs"][e, p]) == inner.trellis.data_ptr()
            assert torch.equal(seen["suh"][p][e], inner.suh) and torch.equal(seen["svh"][p][e], inner.svh)
    assert len(seen["keep"]) == 15


# ---- glmx.hc: the reference's apply_partials / finalize_norm mirror, argument checks (CPU tensors, no launch) ----------

def test_hc_mirror_argument_checks():
    from glmx import hc
    R, D = 2, 256
    x = torch.zeros(R, 4, D)
    fn = torch.zeros(24, 4 * D, dtype=torch.float16)
    part = torch.zeros(R, 4 * D // 128, 25)
    hc.check_mix_args(x, fn, part)                                  # well-formed: no error
    with pytest.raises(ValueError, match="x must be"):
        hc.check_mix_args(torch.zeros(R, 3, D), fn, part)
    with pytest.raises(ValueError, match="D % 128"):
        hc.check_mix_args(torch.zeros(R, 4, 200), fn, part)
    with pytest.raises(ValueError, match="fn must be"):
        hc.check_mix_args(x, fn.float(), part)
    with pytest.raises(ValueError, match="fn must be"):
        hc.check_mix_args(x, torch.zeros(24, 2 * D, dtype=torch.float16), part)
    with pytest.raises(ValueError, match="partials must be"):
        hc.check_mix_args(x, fn, torch.zeros(R, 4 * D // 128, 24))
    with pytest.raises(ValueError, match="y must be"):
        hc.apply_partials(x, torch.zeros(R, D, dtype=torch.bfloat16), torch.zeros(R, 4), torch.zeros(R, 4, 4), fn, part)
    with pytest.raises(ValueError, match="needs post and comb"):
        hc.apply_partials(x, torch.zeros(R, D), None, None, fn, part)
    with pytest.raises(ValueError, match="nw must be"):
        hc.finalize_norm(x, part, torch.zeros(24), torch.zeros(3), torch.zeros(R, 4), torch.zeros(R, 4, 4),
                         torch.zeros(D), torch.zeros(R, D, dtype=torch.float16), 1e-6, 1e-6, 20, 1e-5, 0.0, 1.0)
    with pytest.raises(ValueError, match="out must be"):
        hc.finalize_norm(x, part, torch.zeros(24), torch.zeros(3), torch.zeros(R, 4), torch.zeros(R, 4, 4),
                         torch.zeros(D, dtype=torch.float16), torch.zeros(R, D), 1e-6, 1e-6, 20, 1e-5, 0.0, 1.0)
