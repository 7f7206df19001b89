"""The tier_* API mirror and the exllamav3 hooks on the GPU, through libglmx, against the oracle."""
import numpy as np
import pytest
import torch

from conftest import assert_exact_mode, reference_outputs

pytestmark = pytest.mark.gpu


def _bank_on_device(H=512, I=256, E=8, seed=11):
    from glmx import synth
    bank = synth.make_bank(H, I, E, shared=True, seed=seed)
    tr = torch.from_numpy(bank.trellis).cuda()
    ptrs = torch.tensor([[tr.data_ptr() + bank.proj_offset(e, p) for p in range(3)] for e in range(bank.e_total)],
                        dtype=torch.int64)
    return bank, tr, ptrs


def test_tier_forward_matches_oracle(oracle):
    from glmx import synth, tier
    bank, tr, ptrs = _bank_on_device()
    H, I, E = bank.H, bank.I, bank.E
    s = lambda a, e0, e1: torch.from_numpy(np.ascontiguousarray(a[e0:e1]))
    tier.tier_reset()
    try:
        tier.tier_init(1, [0], None, None, None, None, 1, H, I, 1, 0)
        tier.tier_add_layer(0, ptrs[:E], s(bank.suh[0], 0, E), s(bank.svh[0], 0, E), s(bank.suh[1], 0, E),
                            s(bank.svh[1], 0, E), s(bank.suh[2], 0, E), s(bank.svh[2], 0, E),
                            shared=(ptrs[E], [s(bank.suh[p], E, E + 1)[0] for p in range(3)],
                                    [s(bank.svh[p], E, E + 1)[0] for p in range(3)]))
        x = synth.make_x(4, H, 21)
        sel, w = synth.route_uniform(4, E, 4, 22)
        sel[1, 2] = -1
        xt, st, wt = torch.from_numpy(x.astype(np.float32)), torch.from_numpy(sel), torch.from_numpy(w)
        want = oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=2)
        got = tier.tier_forward(0, xt, st, wt, 2)
        assert got.device.type == "cpu" and got.dtype == torch.float32
        np.testing.assert_array_equal(got.numpy(), want)
        # auto (-1): the reference's rule picks I16 or EXACT; the result is that mode's, bit for bit
        auto = tier.tier_forward(0, xt, st, wt, -1)
        np.testing.assert_array_equal(auto.numpy(), tier.tier_forward(0, xt, st, wt, tier._auto_mode(st, H)).numpy())
        got = tier.tier_forward(0, xt, st, wt, 1).numpy()
        assert_exact_mode(got, oracle.moe_forward(bank, x.astype(np.float32), sel, w, mode=1),
                          *reference_outputs(bank, x, sel, w), label="tier EXACT")
        assert tier.tier_stats()[0] == 4
    finally:
        tier.tier_reset()
    del tr


def test_hooks_with_gpu_layer(oracle):
    """The routing_fn / cpu_split_combine wrappers over a real layer: the partial added into the fp16 MoE output."""
    from glmx import MoELayer, hooks, synth
    bank = synth.make_bank(512, 256, 8, shared=False, seed=12)
    layer = MoELayer.from_bank(bank, device="cuda")
    x = synth.make_x(3, 512, 31)
    sel, w = synth.route_uniform(3, 8, 4, 32)

    class Mod:
        def routing_fn(self, bsz, cfg, z, params):
            return torch.from_numpy(sel).long().cuda(), torch.from_numpy(w).half().cuda()

        def cpu_split_combine(self, fhs, cpu_partial, cpu_pending, shape):
            return fhs

    m = Mod()
    hooks.attach(m, layer, mode=2)
    z = torch.from_numpy(x).cuda()
    so, wo = m.routing_fn(3, None, z, {})
    assert torch.all(so == -1) and torch.all(wo == 0)
    fhs = torch.zeros(3, 512, dtype=torch.float16, device="cuda")
    out = m.cpu_split_combine(fhs, None, None, None).cpu()
    want = oracle.moe_forward(bank, x.astype(np.float32), sel, w.astype(np.float16).astype(np.float32), mode=2)
    np.testing.assert_array_equal(out.numpy(), want.astype(np.float16))


def test_layer_from_exllamav3_matches_bank():
    """The on-disk EXL3 adapter (per-expert trellis tensors, as exllamav3 holds them) gives the same layer as the
    packed bank: bit-identical outputs in both modes."""
    from glmx import MoELayer, hooks, synth
    from test_host_api import fake_exl3_module
    dev = torch.device("cuda", 0)
    bank = synth.make_bank(1024, 512, 6, shared=False, seed=71)
    m = fake_exl3_module(bank, device=dev)
    a = hooks.layer_from_exllamav3(m)
    b = MoELayer.from_bank(bank, device=dev)
    x = torch.from_numpy(synth.make_x(5, 1024, 72)).to(dev)
    s, w = synth.route_uniform(5, 6, 3, 73)
    s, w = torch.from_numpy(s).to(dev), torch.from_numpy(w).to(dev)
    for mode in (1, 2):
        assert torch.equal(a.forward(x, s, w, mode=mode), b.forward(x, s, w, mode=mode)), mode
