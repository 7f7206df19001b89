"""Generates the golden fixtures of tests/golden/ by running the reference's own CPU implementation
(kernels/cpu_avx2/ft_core.h of nkeilar/glm-flash-lite, compiled by oracle/Makefile into oracle/_ref/libftref.so).

Run here, where the reference tree exists:  python tests/golden/make_golden.py
The fixtures hold every input except the trellis bytes, which come from glmx.synth.splitmix_bytes(seed, n) and are
pinned by their SHA-256. Input conventions follow the reference's kernel A/B harness
(tools/bench/kernel-ab-harness.cpp:26-37, 112-132): scales +-(0.5..0.99), x = fp16(0.35 * N(0,1)),
routes (t + 2k) % E with weight 0.25, decode routes (3q + K) % E with weight 0.9 / (q + 1).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "glm-flash-lite_b200"))

from glmx import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402


def bank_splitmix(H, I, E, shared, seed):
    """A harness-style bank whose trellis bytes are the SplitMix64 stream of `seed`."""
    b = synth.make_bank(H, I, E, shared=shared, seed=seed, scale_style="harness")
    b.trellis = synth.splitmix_bytes(seed, b.trellis.size)
    return b


def save_bank(prefix, b, seed, d):
    d[prefix + "H"] = b.H; d[prefix + "I"] = b.I; d[prefix + "E"] = b.E; d[prefix + "shared"] = int(b.shared)
    d[prefix + "seed"] = seed; d[prefix + "trellis_sha256"] = synth.sha256(b.trellis)
    for p in range(3):
        d[f"{prefix}suh{p}"] = b.suh[p]; d[f"{prefix}svh{p}"] = b.svh[p]


def main():
    O.build(ref=True)
    ref = O.Reference()
    ref.start_pool(min(8, os.cpu_count() or 1))
    out = {}

    # 1. decode known answers: random tiles + edge patterns, decoded by the reference's dense_weights
    rnd = synth.splitmix_bytes(101, 60 * 96).reshape(60, 96)
    edge = np.stack([np.zeros(96, np.uint8), np.full(96, 0xFF, np.uint8), np.tile(np.array([0xAA, 0x55], np.uint8), 48),
                     np.arange(96, dtype=np.uint8)])
    tiles = np.concatenate([rnd, edge])
    W = ref.dense(tiles.reshape(-1), 16, 16 * tiles.shape[0])               # one tile row of n tiles
    dec = W.reshape(16, tiles.shape[0], 16).transpose(1, 0, 2).astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "decode_k3.npz"), tiles=tiles, decoded=dec, seed=101)

    # 2. small layer (harness geometry class, H % 512 == 0 as moe_forward's combine phase requires)
    for name, (H, I, E, seed) in {"moe_small": (512, 256, 6, 202), "moe_baseline": (6144, 1536, 4, 303)}.items():
        b = bank_splitmix(H, I, E, True, seed)
        d = {}
        save_bank("", b, seed, d)
        L = ref.layer(b, with_shared=True)
        cases = []
        for nt in (1, 3, 4) if name == "moe_small" else (2,):
            rng = np.random.default_rng(777 + nt)
            x = (0.35 * rng.standard_normal((nt, H))).astype(np.float16).astype(np.float32)
            sel = np.array([[(t + 2 * k) % E for k in range(4)] for t in range(nt)], np.int32)
            w = np.full(sel.shape, 0.25, np.float32)
            cases.append((f"t{nt}", x, sel, w))
        for K in (1, 3):
            rng = np.random.default_rng(991 + K)
            x = (0.35 * rng.standard_normal((1, H))).astype(np.float16).astype(np.float32)
            sel = np.array([[(3 * q + K) % E for q in range(K)]], np.int32)
            w = np.array([[0.9 / (q + 1) for q in range(K)]], np.float32)
            cases.append((f"d{K}", x, sel, w))
        names = []
        for tag, x, sel, w in cases:
            s2, w2 = O.with_shared_routes(sel, w, E)
            d[f"{tag}_x"] = x; d[f"{tag}_sel"] = sel; d[f"{tag}_w"] = w
            d[f"{tag}_exact"] = ref.moe_forward(L, x, s2, w2, mode=1)
            d[f"{tag}_affine"] = ref.moe_forward(L, x, s2, w2, mode=0)
            d[f"{tag}_band_exact"] = ref.moe_forward(L, x, s2, w2, mode=1, band=True)
            d[f"{tag}_expert0_fp64"] = ref.expert_fp64(L, int(sel[0, 0]), x[0])
            d[f"{tag}_shared_fp64"] = ref.expert_fp64(L, E, x[0])
            names.append(tag)
        d["cases"] = np.array(names)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **d)
    # 3. I16 mode (the reference's mode 2) at the reference's own geometry H=4096, I=2048, where its scratch is valid
    #    (ft_core.h:1353). Single-pick routes (weight 1) make the layer output equal one expert's output, so the pin is
    #    bit-exact; a multi-pick case checks the combine.
    H, I, E, seed = 4096, 2048, 5, 404
    b = bank_splitmix(H, I, E, False, seed)
    d = {}
    save_bank("", b, seed, d)
    L = ref.layer(b, with_shared=False)
    rng = np.random.default_rng(4242)
    x = (0.35 * rng.standard_normal((E, H))).astype(np.float16).astype(np.float32)
    sel = np.arange(E, dtype=np.int32).reshape(E, 1)
    w = np.ones((E, 1), np.float32)
    d["single_x"] = x; d["single_sel"] = sel; d["single_w"] = w
    d["single_i16"] = ref.moe_forward(L, x, sel, w, mode=2)
    sel2 = np.array([[(t + 2 * k) % E for k in range(3)] for t in range(3)], np.int32)
    w2 = np.array([[0.5, 0.3, 0.2]] * 3, np.float32)
    d["multi_x"] = x[:3]; d["multi_sel"] = sel2; d["multi_w"] = w2
    d["multi_i16"] = ref.moe_forward(L, x[:3], sel2, w2, mode=2)
    np.savez_compressed(os.path.join(HERE, "moe_i16_h4096.npz"), **d)
    ref.stop_pool()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
