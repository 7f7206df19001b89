"""The reference's expert-tier extension API, backed by libglmx on the GPU.

Mirrors the pybind module of kernels/cpu_avx2/ft_tier_ext.cpp (1288-1334): same function names, argument order and
meaning, same argument checks and messages (RuntimeError, as TORCH_CHECK raises). Differences, all because the experts
live in HBM instead of a pinned host arena served by a CPU worker:

* tier_init's threads / cpus / ctrl / hx / picks / hout / swz describe the CPU worker and its mapped buffers; they are
  accepted and ignored (there is no worker, no handshake and no block-contiguous CPU copy).
* tier_add_layer's `ptrs` [E, 3] are device addresses of the native-layout gate / up / down trellis tensors (the
  HBM-resident copies exllamav3 already holds, glm53/expert_cache.py:603-616), not host addresses.
* tier_forward runs on the GPU. Mode -1 (auto) follows the reference's rule (ft_tier_ext.cpp:899-900): I16 when no
  expert has more than 2 of the call's tokens, where the reference's I16 is valid (H <= 4096, its scratch limit,
  ft_core.h:1353); otherwise EXACT, in place of the reference's AFFINE, which is a CPU shortcut with no GPU kernel here.
  Mode 0 (AFFINE) is rejected.
  The result is returned on x's device (a CPU x gets a CPU result, as in the reference).
"""
from __future__ import annotations

import time

import torch

from .layer import MoELayer

_MODES = {-1: None, 1: 1, 2: 2}


def _auto_mode(sel: torch.Tensor, H: int) -> int:
    """tier_forward's mode -1: I16 for <= 2 tokens per expert at H <= 4096 (the reference's rule and range), else EXACT."""
    s = sel[sel >= 0]
    most = int(torch.bincount(s.reshape(-1).long()).max()) if s.numel() else 0
    return 2 if most <= 2 and H <= 4096 else 1


class _Tier:
    def __init__(self, mode: int, H: int, I: int, nlayers: int):
        self.mode, self.H, self.I = int(mode), int(H), int(I)
        self.layers: list = [None] * int(nlayers)
        self.running = False
        self.act_limit = 0.0
        self.stats = dict(jobs=0, experts=0, tokens=0, empty=0, busy_ns=0)


T: _Tier | None = None


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def tier_init(threads, cpus, ctrl, hx, picks, hout, mode, H, I, nlayers, swz) -> None:
    """ft_tier_ext.cpp:137-157. Only mode, H, I and nlayers are used."""
    global T
    _check(T is None, "tier already initialised")
    _check(int(H) % 128 == 0 and int(I) % 128 == 0, "H and I must be multiples of 128")
    T = _Tier(mode, H, I, nlayers)


def tier_add_layer(li, ptrs, suh_g, svh_g, suh_u, svh_u, suh_d, svh_d, shared=None, bits=(3, 3, 3)) -> None:
    """ft_tier_ext.cpp:160-183. ptrs: int64 [E, 3] device addresses; scales fp16 [E, k] / [E, n] (CPU or CUDA).
    shared (extension): optional (ptrs [3], suh (3 x [k]), svh (3 x [n])) of an always-on shared expert."""
    _check(T is not None, "init first")
    E = int(ptrs.shape[0])
    H, I = T.H, T.I
    for t in (suh_g, svh_g, suh_u, svh_u, suh_d, svh_d):
        _check(t.dtype == torch.float16 and t.is_contiguous() and t.shape[0] == E, "scales: CPU fp16 contiguous [E, .]")
    _check(suh_g.shape[1] == H and svh_g.shape[1] == I and suh_d.shape[1] == I and svh_d.shape[1] == H, "scale shapes")
    _check(0 <= int(li) < len(T.layers), "layer index out of range")
    suh = [suh_g, suh_u, suh_d]
    svh = [svh_g, svh_u, svh_d]
    p = torch.as_tensor(ptrs, dtype=torch.int64).cpu()
    if shared is not None:
        sp, ss, sv = shared
        p = torch.cat([p, torch.as_tensor(sp, dtype=torch.int64).reshape(1, 3)])
        suh = [torch.cat([a.to(b.device), b.reshape(1, -1).to(a.device)]) for a, b in zip(suh, ss)]
        svh = [torch.cat([a.to(b.device), b.reshape(1, -1).to(a.device)]) for a, b in zip(svh, sv)]
    T.layers[int(li)] = MoELayer(H, I, E, p, suh, svh, bits=bits, has_shared=shared is not None, act_limit=T.act_limit,
                                 keep=[ptrs])


def tier_start(cpu0=0) -> None:
    """ft_tier_ext.cpp:814-845: starts the CPU worker. Here only the running flag (tier_forward refuses while set)."""
    _check(T is not None, "init first")
    T.running = True


def tier_stop() -> None:
    if T is not None:
        T.running = False


def tier_reset() -> None:
    """Drop all state (tests)."""
    global T
    T = None


def tier_forward(li, x: torch.Tensor, sel: torch.Tensor, w: torch.Tensor, mode: int) -> torch.Tensor:
    """ft_tier_ext.cpp:865-904: x fp32 [m, H], sel int32 [m, k], w fp32 [m, k] -> fp32 [m, H] (sel < 0 skipped)."""
    _check(T is not None and not T.running, "tier_forward: worker running")
    _check(0 <= int(li) < len(T.layers) and T.layers[int(li)] is not None, "tier_forward: layer not registered")
    _check(int(mode) in _MODES, "tier_forward: mode 0 (AFFINE) has no GPU kernel; use -1, 1 (EXACT) or 2 (I16)")
    layer = T.layers[int(li)]
    _check(x.dim() == 2 and x.shape[1] == T.H, "tier_forward: x must be [m, H]")
    dev = layer.device
    t0 = time.perf_counter_ns()
    m = _MODES[int(mode)] if int(mode) != -1 else _auto_mode(sel, T.H)
    out = layer.forward(x.to(dev, non_blocking=True), sel.to(dev, torch.int32), w.to(dev, torch.float32), mode=m)
    res = out.to(x.device)
    T.stats["busy_ns"] += time.perf_counter_ns() - t0
    T.stats["jobs"] += 1
    T.stats["tokens"] += int(x.shape[0])
    T.stats["experts"] += int(torch.unique(sel[sel >= 0]).numel()) if sel.numel() else 0
    return res


def tier_stats() -> list:
    """ft_tier_ext.cpp:906-914 (first six entries: jobs, experts, tokens, empty, busy_ns, swz_bytes)."""
    if T is None:
        return []
    s = T.stats
    return [s["jobs"], s["experts"], s["tokens"], s["empty"], s["busy_ns"], 0]


def tier_set_act_limit(limit: float) -> None:
    """ft_tier_ext.cpp:635: SwiGLU clamp for every registered layer (0 = off)."""
    _check(T is not None, "init first")
    T.act_limit = float(limit)
    for layer in T.layers:
        if layer is not None:
            layer.set_act_limit(limit)
