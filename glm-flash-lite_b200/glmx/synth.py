"""Seeded synthetic inputs for the routed-expert MoE layer (the BASELINE configs use synthetic data).

Two generators:

* ``splitmix_bytes(seed, n)`` - a counter-based SplitMix64 byte stream written with plain uint64 arithmetic, so the
  same seed gives the same bytes on every machine and numpy version. The golden fixtures under tests/golden/ store
  only the seed and a SHA-256 of the trellis bytes they were made from.
* numpy ``default_rng`` draws for the bulk synthetic banks of the benchmark (value distributions of BASELINE.json:
  uniform trellis bytes, +-1 Hadamard signs, svh ~ sign * |N(0.02, 0.005)|, activations ~ N(0, 1)).

Any 32*K bytes form a valid EXL3 trellis tile (tools/bench/kernel-ab-harness.cpp:1 of the reference), so uniform
random bytes are a faithful stand-in for quantised experts.
"""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

_GOLDEN_GAMMA = np.uint64(0x9E3779B97F4A7C15)


def splitmix_u64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """n SplitMix64 outputs of the counter stream seed + (offset + i + 1) * gamma."""
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * _GOLDEN_GAMMA
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def splitmix_bytes(seed: int, n: int) -> np.ndarray:
    words = splitmix_u64(seed, (n + 7) // 8)
    return words.view(np.uint8)[:n].copy()


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def matrix_bytes(k: int, n: int, bits: int) -> int:
    """Bytes of one EXL3 trellis tensor [k x n]: (k/16)(n/16) tiles of 32*bits bytes."""
    assert k % 16 == 0 and n % 16 == 0 and bits in (2, 3, 4)
    return (k // 16) * (n // 16) * 32 * bits


@dataclasses.dataclass
class ExpertBank:
    """Host copy of E experts (+ optional shared expert, stored as the last expert) in the packed bank layout:
    per expert gate | up | down trellis bytes, experts contiguous. Scales follow tier_add_layer's shapes
    (ft_tier_ext.cpp:160-183): suh/svh fp16 [E, k] / [E, n] per projection."""
    H: int
    I: int
    E: int                      # routed experts
    shared: bool
    bits: tuple                 # (gate, up, down) bits per weight
    trellis: np.ndarray         # uint8 [E_total * expert_bytes]
    suh: list                   # 3 x fp16 [E_total, k]
    svh: list                   # 3 x fp16 [E_total, n]

    @property
    def e_total(self) -> int:
        return self.E + (1 if self.shared else 0)

    def proj_bytes(self, p: int) -> int:
        k, n = ((self.H, self.I), (self.H, self.I), (self.I, self.H))[p]
        return matrix_bytes(k, n, self.bits[p])

    @property
    def expert_bytes(self) -> int:
        return sum(self.proj_bytes(p) for p in range(3))

    def proj_offset(self, e: int, p: int) -> int:
        return e * self.expert_bytes + sum(self.proj_bytes(q) for q in range(p))

    def proj(self, e: int, p: int) -> np.ndarray:
        o = self.proj_offset(e, p)
        return self.trellis[o:o + self.proj_bytes(p)]


def _half(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16)


def make_bank(H: int, I: int, E: int, shared: bool = True, bits=(3, 3, 3), seed: int = 0,
              scale_style: str = "baseline") -> ExpertBank:
    """scale_style 'baseline': suh = +-1, svh = sign * |N(0.02, 0.005)|.
    'harness': suh, svh = +-(0.5 .. 0.99) (tools/bench/kernel-ab-harness.cpp:29-37 of the reference)."""
    bits = tuple(int(b) for b in bits)
    et = E + (1 if shared else 0)
    rng = np.random.default_rng(seed)
    per = sum(matrix_bytes(k, n, b) for (k, n), b in zip(((H, I), (H, I), (I, H)), bits))
    trellis = rng.integers(0, 256, size=et * per, dtype=np.uint8)
    dims = ((H, I), (H, I), (I, H))
    suh, svh = [], []
    for (k, n) in dims:
        if scale_style == "baseline":
            suh.append(_half(np.where(rng.random((et, k)) < 0.5, -1.0, 1.0)))
            mag = np.abs(rng.normal(0.02, 0.005, size=(et, n)))
            svh.append(_half(np.where(rng.random((et, n)) < 0.5, -mag, mag)))
        else:
            def hs(shape):
                sgn = np.where(rng.integers(0, 2, size=shape) == 1, 1.0, -1.0)
                return _half(sgn * (0.5 + 0.01 * rng.integers(0, 50, size=shape)))
            suh.append(hs((et, k)))
            svh.append(hs((et, n)))
    return ExpertBank(H, I, E, shared, bits, trellis, suh, svh)


def make_x(ntok: int, H: int, seed: int, scale: float = 1.0) -> np.ndarray:
    """fp16 activations ~ scale * N(0, 1), returned as fp16."""
    rng = np.random.default_rng(seed)
    return _half(scale * rng.standard_normal((ntok, H)))


def route_uniform(ntok: int, E: int, topk: int, seed: int):
    """Router of BASELINE configs[1]: fp32 logits ~ N(0,1) over E experts, sigmoid gates, top-k, renormalised to
    sum 1. Returns (sel int32 [ntok, topk], w fp32 [ntok, topk])."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((ntok, E)).astype(np.float32)
    gates = 1.0 / (1.0 + np.exp(-logits))
    sel = np.argsort(-gates, axis=1, kind="stable")[:, :topk].astype(np.int32)
    w = np.take_along_axis(gates, sel, axis=1)
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return sel, w


def route_zipf(ntok: int, E: int, topk: int, s: float, seed: int):
    """expert popularity Zipf(s) over a seeded permutation of the E experts, top-k without
    replacement (Gumbel-top-k on log p). Weights: renormalised sigmoid of N(0,1) logits."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    logp = np.empty(E)
    logp[perm] = np.log(p / p.sum())
    g = rng.gumbel(size=(ntok, E)) + logp[None, :]
    sel = np.argsort(-g, axis=1, kind="stable")[:, :topk].astype(np.int32)
    gates = 1.0 / (1.0 + np.exp(-rng.standard_normal((ntok, topk))))
    w = (gates / gates.sum(axis=1, keepdims=True)).astype(np.float32)
    return sel, w


def route_hotset(ntok: int, E: int, topk: int, hot: int, frac: float, seed: int):
    """BASELINE configs[4] hot-set skew: `hot` experts receive about `frac` of the assignments."""
    rng = np.random.default_rng(seed)
    hot_ids = rng.permutation(E)[:hot]
    p = np.full(E, (1.0 - frac) / (E - hot))
    p[hot_ids] = frac / hot
    g = rng.gumbel(size=(ntok, E)) + np.log(p)[None, :]
    sel = np.argsort(-g, axis=1, kind="stable")[:, :topk].astype(np.int32)
    gates = 1.0 / (1.0 + np.exp(-rng.standard_normal((ntok, topk))))
    w = (gates / gates.sum(axis=1, keepdims=True)).astype(np.float32)
    return sel, w


def unique_experts(sel: np.ndarray, E: int) -> int:
    s = sel[(sel >= 0) & (sel < E)]
    return int(np.unique(s).size)


def router_inputs(ntok: int, E: int, seed: int, logit_scale: float = 6.0, bias_scale: float = 0.5):
    """Router test inputs from the SplitMix64 stream of `seed` (no RNG library involved, so every machine makes the
    same values): fp32 logits uniform in +-logit_scale/2 at 24-bit resolution [ntok, E] and a score-correction bias
    uniform in +-bias_scale/2 [E]."""
    u = (splitmix_u64(seed, ntok * E + E) >> np.uint64(40)).astype(np.float64) / float(1 << 24)
    logits = (logit_scale * (u[: ntok * E] - 0.5)).astype(np.float32).reshape(ntok, E)
    bias = (bias_scale * (u[ntok * E:] - 0.5)).astype(np.float32)
    return logits, bias
