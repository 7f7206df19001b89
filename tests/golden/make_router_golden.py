"""Generates tests/golden/router.npz: the GLM-4 MoE routing as the published model code computes it
(transformers 5.5, models/glm4_moe/modeling_glm4_moe.py: Glm4MoeTopkRouter.forward 302-305 for the gate,
Glm4MoeMoE.route_tokens_to_experts 389-412 for the selection). The reference takes its router from exllamav3
(un-vendored, v1.5.1), which implements the same published routing; transformers is installed in this image and is the
executable statement of it used to pin the router restatement in oracle/ft_oracle.c.

Run:  python tests/golden/make_router_golden.py
Inputs come from glmx.synth.router_inputs (SplitMix64, no RNG library); the fixture stores the picks as sorted expert
ids per token (torch.topk with sorted=False leaves the order open) with their weights, and the gate case's logits.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "glm-flash-lite_b200"))

from glmx import synth  # noqa: E402

# name: (ntok, E, topk, n_group, topk_group, norm, scale, with_bias, seed)
CASES = {
    "glm288": (64, 288, 8, 1, 1, True, 1.0, True, 7001),        # BASELINE routing: 288 experts, top-8, renormalised
    "grouped256": (32, 256, 8, 8, 4, True, 2.5, True, 7002),    # group-limited: 8 groups, best 4 kept
    "nonorm160": (32, 160, 8, 1, 1, False, 2.5, False, 7003),   # no renormalisation, scaling factor only
}
GATE = dict(ntok=16, H=512, E=288, seed=7004)                   # gate linear: bf16 z and W, fp32 logits


def gate_inputs(ntok, H, E, seed):
    """bf16-valued z [ntok, H] and W [E, H] (as fp32 arrays) from SplitMix64."""
    u = (synth.splitmix_u64(seed, ntok * H + E * H) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    to_bf16 = lambda a: (np.asarray(a, np.float32).view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)
    z = to_bf16(4.0 * (u[: ntok * H] - 0.5)).reshape(ntok, H)
    W = to_bf16(0.1 * (u[ntok * H:] - 0.5)).reshape(E, H)
    return z, W


def _route(logits, bias, topk, n_group, topk_group, norm, scale):
    import torch
    from transformers.models.glm4_moe.modeling_glm4_moe import Glm4MoeMoE
    E = logits.shape[1]
    me = types.SimpleNamespace(gate=types.SimpleNamespace(e_score_correction_bias=torch.from_numpy(bias)),
                               n_group=n_group, n_routed_experts=E, topk_group=topk_group, top_k=topk,
                               norm_topk_prob=norm, routed_scaling_factor=scale)
    idx, w = Glm4MoeMoE.route_tokens_to_experts(me, torch.from_numpy(logits))
    idx, w = idx.numpy().astype(np.int32), w.numpy().astype(np.float32)
    order = np.argsort(idx, axis=1, kind="stable")
    return np.take_along_axis(idx, order, 1), np.take_along_axis(w, order, 1)


def main():
    import torch
    out = {}
    for name, (ntok, E, topk, ng, tg, norm, scale, wb, seed) in CASES.items():
        logits, bias = synth.router_inputs(ntok, E, seed)
        if not wb:
            bias = np.zeros(E, np.float32)
        out[name + "_sel"], out[name + "_w"] = _route(logits, bias, topk, ng, tg, norm, scale)
    z, W = gate_inputs(**GATE)
    logits = torch.nn.functional.linear(torch.from_numpy(z).to(torch.bfloat16).float(),
                                        torch.from_numpy(W).to(torch.bfloat16).float()).numpy()
    out["gate_logits"] = logits.astype(np.float32)
    out["gate_sel"], out["gate_w"] = _route(logits, np.zeros(GATE["E"], np.float32), 8, 1, 1, True, 1.0)
    np.savez_compressed(os.path.join(HERE, "router.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
