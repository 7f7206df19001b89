"""Drop-in for the reference's monkeypatch hooks on exllamav3's BlockSparseMLP (glm53/cpu_tier.py:305-351).

The reference wraps two methods of every MoE module:
  routing_fn(bsz, cfg, z, params) -> (sel int64 [bsz, k], w fp16 [bsz, k])   ft_split then hands the picks the CPU tier
      takes back with id -1 / weight 0 (or the id kept with weight 0 when keep_ids), so exllamav3's own experts skip them
  cpu_split_combine(fhs, cpu_partial, cpu_pending, shape) -> fhs            ft_combine adds the tier's fp32 partial into
      the MoE output (fp16: half(float(o) + v), ft_tier_cu.cu:226-233) before the stock combine runs
Here the tier is the whole routed-expert computation on the GPU: `attach` takes every pick (so exllamav3's expert
kernels see only masked picks), runs glmx on the same stream right after routing, and adds its result in
cpu_split_combine, keeping both method signatures and the masking conventions.
"""
from __future__ import annotations

import torch

from .layer import MoELayer


def attach(module, layer: MoELayer, mode: int = 1, max_bsz: int | None = None) -> None:
    """Wrap module.routing_fn and module.cpu_split_combine to route every pick through `layer`. mode 1 EXACT (default:
    the exact-mode arithmetic of exllamav3's expert forward), 2 I16 (bit-identical to the reference's CPU I16 kernel)."""
    orig_route = module.routing_fn
    orig_comb = module.cpu_split_combine
    module._glmx_pending = None

    def routed(bsz, cfg, z, params, _orig=orig_route, _m=module):
        sel, w = _orig(bsz, cfg, z, params)
        _m._glmx_pending = None
        if (max_bsz is not None and bsz > max_bsz) or params.get("autosplit_measure") or params.get("tp_warmup"):
            return sel, w                                  # the reference's bypass conditions (cpu_tier.py:315-317)
        zz = z.view(bsz, -1)
        if zz.dtype != torch.half or not zz.is_contiguous():
            zz = zz.half().contiguous()
        _m._glmx_pending = layer.forward(zz, sel.reshape(bsz, -1), w.reshape(bsz, -1), mode=mode)
        keep_ids = bsz > 8                                 # ft_tier_cu.cu:131-140: ids kept, weight 0 for bsz > 8
        sel_out = sel if keep_ids else torch.full_like(sel, -1)
        return sel_out, torch.zeros_like(w)

    def comb(fhs, cpu_partial, cpu_pending, shape, _orig=orig_comb, _m=module):
        p = _m._glmx_pending
        if p is not None:
            _m._glmx_pending = None
            f = fhs if fhs.is_contiguous() else fhs.contiguous()
            v = p.view(f.shape)
            if f.dtype == torch.float16:
                f.copy_((f.float() + v).half())
            else:
                f.add_(v.to(f.dtype))
            fhs = f
        return _orig(fhs, cpu_partial, cpu_pending, shape)

    module.routing_fn = routed
    module.cpu_split_combine = comb


def layer_from_exllamav3(module, device=None) -> MoELayer:
    """Build a MoELayer from an exllamav3 BlockSparseMLP's HBM-resident expert tensors: multi_gate / multi_up /
    multi_down .linears[e].inner.{trellis, suh, svh} (the attributes cpu_tier.start reads, glm53/cpu_tier.py:535-537).
    The shared expert (module.shared_experts) stays with exllamav3 (the reference overlaps it on a side stream,
    glm53/k_overlap.py:63-88)."""
    g, u, d = module.multi_gate.linears, module.multi_up.linears, module.multi_down.linears
    E = len(g)
    ptrs = torch.tensor([[g[e].inner.trellis.data_ptr(), u[e].inner.trellis.data_ptr(), d[e].inner.trellis.data_ptr()]
                         for e in range(E)], dtype=torch.int64)
    stack = lambda lins, attr: torch.stack([getattr(l.inner, attr).view(-1) for l in lins]).half().contiguous()
    suh = [stack(g, "suh"), stack(u, "suh"), stack(d, "suh")]
    svh = [stack(g, "svh"), stack(u, "svh"), stack(d, "svh")]
    keep = [l.inner.trellis for lins in (g, u, d) for l in lins]
    return MoELayer(module.hidden_size, module.intermediate_size, E, ptrs, suh, svh, has_shared=False,
                    act_limit=float(getattr(module, "act_limit", 0.0) or 0.0), keep=keep,
                    device=device or g[0].inner.trellis.device)
