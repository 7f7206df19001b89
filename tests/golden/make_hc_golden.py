"""Writes tests/golden/hc_ref.npz: outputs of the reference's own fused hyper-connection kernels (glm53/k_hcfuse.py,
`apply_partials` = hc_apply of the previous site + hc_mix_partials of this one, and `finalize_norm` = hc_mix_finalize
with Sinkhorn + the site's RMSNorm) on seeded inputs, for pinning the oracle's and the GPU's hc code.

The kernels are the reference's source built by oracle/build_hc_ref.py (run in a container that holds the reference
tree); this script needs a CUDA device and that prebuilt module, and no reference tree:
    python tests/golden/make_hc_golden.py [out.npz]

Inputs (stated here, stored in the file too): x stream stacks N(0, 1) fp32 [R, 4, D]; y N(0, 1) as fp16 or fp32;
post = 2 sigmoid(N(0, 1)); comb rows of a random positive matrix normalised to sum 1 per column; fn N(0, 1) * 0.02
as fp16 [24, 4D]; finalize: base N(0, 1) * 0.5 [24], scale [0.5, 1, 1.5], norm weight N(1, 0.1) in bf16 or fp16.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

APPLY_CASES = [("apply_h", 3, 512, "half", 11), ("apply_f", 2, 768, "float", 12), ("mix_only", 3, 512, None, 13)]
# (name, R, D, norm weight dtype, cbias, cscale); finalize_norm is built for 64 partial chunks: D = 4096
FINAL_CASES = [("final_h", 2, 4096, "half", 0.0, 1.0, 21), ("final_b", 3, 4096, "bfloat16", 1.0, 0.5, 22)]
RMS_EPS, HC_EPS, ITERS, N_EPS = 1e-6, 1e-6, 20, 1e-5


def inputs_apply(R, D, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, 4, D)).astype(np.float32)
    y = rng.standard_normal((R, D)).astype(np.float32)
    post = (2.0 / (1.0 + np.exp(-rng.standard_normal((R, 4))))).astype(np.float32)
    m = rng.random((R, 4, 4)) + 0.05
    comb = (m / m.sum(axis=1, keepdims=True)).astype(np.float32)
    fn = (rng.standard_normal((24, 4 * D)) * 0.02).astype(np.float16)
    return x, y, post, comb, fn


def inputs_final(R, D, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, 4, D)).astype(np.float32)
    fn = (rng.standard_normal((24, 4 * D)) * 0.02).astype(np.float16)
    base = (rng.standard_normal(24) * 0.5).astype(np.float32)
    scale = np.array([0.5, 1.0, 1.5], np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return x, fn, base, scale, nw


def main(out_path):
    import torch

    from oracle.build_hc_ref import load_built
    k = load_built()
    dev = torch.device("cuda", 0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    res = {}
    for name, R, D, ydt, seed in APPLY_CASES:
        x, y, post, comb, fn = inputs_apply(R, D, seed)
        xt = t(x)
        part = torch.zeros((R, 4 * D // 128, 25), dtype=torch.float32, device=dev)
        if ydt is None:
            k.apply_partials(xt, None, None, None, t(fn), part)
        else:
            yt = t(y).half() if ydt == "half" else t(y)
            k.apply_partials(xt, yt, t(post), t(comb), t(fn), part)
            y = yt.float().cpu().numpy()
        torch.cuda.synchronize()
        res.update({f"{name}_x": x, f"{name}_y": y, f"{name}_post": post, f"{name}_comb": comb, f"{name}_fn": fn,
                    f"{name}_xout": xt.cpu().numpy(), f"{name}_part": part.cpu().numpy()})
    for name, R, D, wdt, cbias, cscale, seed in FINAL_CASES:
        x, fn, base, scale, nw = inputs_final(R, D, seed)
        xt = t(x)
        part = torch.zeros((R, 4 * D // 128, 25), dtype=torch.float32, device=dev)
        k.apply_partials(xt, None, None, None, t(fn), part)
        post = torch.zeros((R, 4), dtype=torch.float32, device=dev)
        comb = torch.zeros((R, 4, 4), dtype=torch.float32, device=dev)
        out = torch.zeros((R, D), dtype=torch.float16, device=dev)
        nwt = t(nw).to(torch.bfloat16 if wdt == "bfloat16" else torch.float16)
        k.finalize_norm(xt, part, t(base), t(scale), post, comb, nwt, out, RMS_EPS, HC_EPS, ITERS, N_EPS, cbias, cscale)
        torch.cuda.synchronize()
        res.update({f"{name}_x": x, f"{name}_part": part.cpu().numpy(), f"{name}_base": base, f"{name}_scale": scale,
                    f"{name}_nw": nwt.float().cpu().numpy(), f"{name}_post": post.cpu().numpy(),
                    f"{name}_comb": comb.cpu().numpy(), f"{name}_out": out.cpu().numpy(),
                    f"{name}_args": np.array([RMS_EPS, HC_EPS, ITERS, N_EPS, cbias, cscale], np.float64)})
    np.savez_compressed(out_path, **res)
    print("wrote", out_path, sorted(res))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "hc_ref.npz"))
